// Stage 3 (tensor-core path): masked attention on tcgen05 / TMEM for bf16 or
// fp16 Q/K/V with DQ == DV in {64, 128}.
//
//   O[b,t,h,:] = softmax_{s in keep(t)}(scale * <Q[b,t,h,:], K[b,s,h,:]>) @ V[b,s,h,:]
//   keep(t)    = { s <= t : scores[b,t,s] >= thr[b,t] }
//
// This is the reference's threshold form, sparse_attention_with_threshold
// (dsa_attention.py:230-324): a causal flash attention in which every logit
// whose indexer score is below the row's top-K threshold is dropped.  The
// kept set arrives as a bitmap (one bit per (query row, key), built by
// kept_bitmap_kernel from scores and thr), so each 128x128 tile's mask is
// four 32-bit words per query row.  Scanning the causal keys on the tensor
// cores does ~T/(2k) times the FLOPs of a gather over the kept keys, but the
// K/V tiles are shared by 128 query rows instead of being re-read per row,
// which the gather form cannot do: the gather's bytes (HQ*(DQ+DV)*2 per kept
// key per row) are L1-throughput bound far below this kernel's rate.
//
// Persistent, warp-specialised, one CTA per SM, one work unit = (batch,
// 128-row query tile, head); units are dealt longest first:
//   warp 0      TMA producer: the unit's Q tile once, then per key block
//               K[s0:s0+128, h, :] and V[s0:s0+128, h, :] (128-byte swizzle,
//               no multicast) through two mbarrier rings
//   warp 1      MMA issuer (one thread): S_j = Q K_j^T (M=128, N=128) into one
//               of two TMEM buffers, one block ahead of the softmax; then
//               O += P_j V_j (M=128, N=D, V read MN-major) into a TMEM
//               accumulator that lives for the whole unit
//   warps 2..5  softmax (one thread per query row): tcgen05.ld of S_j, mask,
//               online softmax in the exp2 domain with lazy rescaling (O in
//               TMEM is rescaled only when the row max grows by more than 2^8),
//               P_j written to shared memory as bf16/fp16 in the MMA's swizzled
//               K-major layout; after the last block O / l is stored as fp32
// Every mbarrier wait is bounded (2 s of device time); on timeout the CTA's
// warps leave their loops, TMEM is freed, and a device flag records it for
// dsa_device_status().
#include <cuda.h>
#include <math.h>
#include <stdio.h>
#include <stdlib.h>

#include "common.cuh"
#include "tc_ptx.cuh"

namespace dsa {

__device__ int g_attn_tc_timeout = 0;

namespace {

using namespace tc;

constexpr int BM = 128;                       // query rows per tile (TMEM lanes)
constexpr int BN = 128;                       // keys per block
constexpr int SM_WARPS = 4;                   // softmax warps
constexpr int NTHREADS = 64 + SM_WARPS * 32;
constexpr uint32_t TMEM_COLS = 512;           // S buffers at 0 and 128, O at 256
constexpr uint32_t OCOL = 256;
constexpr uint32_t PBYTES = BM * BN * 2;      // one P tile (16-bit)
constexpr float kNegInf = -INFINITY;

struct AtParams {
    float* O;
    const uint32_t* bits;
    int64_t words;        // bitmap words per query row (multiple of 4)
    int64_t T_q, T_k, q_row0;
    int B, HQ, D;
    int n_qt, nkb, total_units;
    int nK, nV, nP;
    uint32_t q_bytes, kv_bytes;
    float sl2;            // scale * log2(e)
    int stall;            // test hook: the producer issues no loads, so every wait times out
    int o_vec8;           // O 32-byte aligned: 256-bit output stores
    unsigned long long timeout_ns;
};

struct Unit {
    int b, h, qt, nblk;
};

// unit index -> (batch, head, query tile); the longest tiles (most key
// blocks) come first so the round-robin deal ends balanced
__device__ __forceinline__ Unit decode_unit(int u, const AtParams& p) {
    Unit r;
    const int bh = p.B * p.HQ;
    const int qr = u / bh, rem = u - qr * bh;
    r.qt = p.n_qt - 1 - qr;
    r.b = rem / p.HQ;
    r.h = rem - r.b * p.HQ;
    int64_t tq_end = (int64_t)(r.qt + 1) * BM;
    if (tq_end > p.T_q) tq_end = p.T_q;
    int64_t nb = (p.q_row0 + tq_end - 1) / BN + 1;
    if (nb > p.nkb) nb = p.nkb;
    r.nblk = (int)nb;
    return r;
}

__device__ __forceinline__ uint32_t pack2(float a, float b, bool f16) {
    if (f16) {
        const __half2 h = __floats2half2_rn(a, b);
        return *reinterpret_cast<const uint32_t*>(&h);
    }
    const __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<const uint32_t*>(&h);
}

template <bool F16>
__global__ void __launch_bounds__(NTHREADS, 1)
    attn_tc_kernel(const __grid_constant__ CUtensorMap tmq, const __grid_constant__ CUtensorMap tmk,
                   const __grid_constant__ CUtensorMap tmv, const AtParams p) {
    extern __shared__ uint8_t smem_raw[];
    __shared__ uint32_t tmem_slot;
    __shared__ int s_abort;
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                               ~uintptr_t(1023));
    // V is followed by P, so every operand region lies inside the allocation
    uint8_t* sQ = smem;
    uint8_t* sK = sQ + p.q_bytes;
    uint8_t* sV = sK + (size_t)p.nK * p.kv_bytes;
    uint8_t* sP = sV + (size_t)p.nV * p.kv_bytes;
    uint64_t* q_full = reinterpret_cast<uint64_t*>(sP + (size_t)p.nP * PBYTES);
    uint64_t* q_empty = q_full + 1;
    uint64_t* k_full = q_empty + 1;
    uint64_t* k_empty = k_full + p.nK;
    uint64_t* v_full = k_empty + p.nK;
    uint64_t* v_empty = v_full + p.nV;
    uint64_t* s_full = v_empty + p.nV;   // [2] S_j in TMEM buffer j&1
    uint64_t* s_free = s_full + 2;       // [2] softmax has read it
    uint64_t* p_full = s_free + 2;       // [2] P_j in shared buffer j%nP
    uint64_t* pv_done = p_full + 2;      // [2] O += P_j V_j done, by parity of j

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nch = p.D / 64;            // 128-byte chunks per Q/K/V row
    int* flag = &g_attn_tc_timeout;

    if (threadIdx.x == 32) {
        s_abort = 0;
        mbar_init(q_full, 1);
        mbar_init(q_empty, 1);
        for (int s = 0; s < p.nK; ++s) {
            mbar_init(&k_full[s], 1);
            mbar_init(&k_empty[s], 1);
        }
        for (int s = 0; s < p.nV; ++s) {
            mbar_init(&v_full[s], 1);
            mbar_init(&v_empty[s], 1);
        }
        for (int s = 0; s < 2; ++s) {
            mbar_init(&s_full[s], 1);
            mbar_init(&s_free[s], SM_WARPS);
            mbar_init(&p_full[s], SM_WARPS);
            mbar_init(&pv_done[s], 1);
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
            int ks = 0, vs = 0;
            uint32_t kph = 0, vph = 0, qph = 0;
            bool ok = true;
            for (int u = blockIdx.x; ok && u < p.total_units; u += gridDim.x) {
                const Unit w = decode_unit(u, p);
                if (!(ok = mbar_wait(q_empty, qph ^ 1, &s_abort, p.timeout_ns, flag))) break;
                qph ^= 1;
                if (!p.stall) {
                    mbar_expect_tx(q_full, p.q_bytes);
                    for (int c = 0; c < nch; ++c)
                        tma_load_4d(sQ + c * BM * 128, &tmq, q_full, c * 64, w.h, w.qt * BM, w.b);
                }
                for (int j = 0; j < w.nblk; ++j) {
                    if (!(ok = mbar_wait(&k_empty[ks], kph ^ 1, &s_abort, p.timeout_ns, flag))) break;
                    if (!p.stall) {
                        mbar_expect_tx(&k_full[ks], p.kv_bytes);
                        for (int c = 0; c < nch; ++c)
                            tma_load_4d(sK + (size_t)ks * p.kv_bytes + c * BN * 128, &tmk, &k_full[ks],
                                        c * 64, w.h, j * BN, w.b);
                    }
                    if (++ks == p.nK) { ks = 0; kph ^= 1; }
                    if (!(ok = mbar_wait(&v_empty[vs], vph ^ 1, &s_abort, p.timeout_ns, flag))) break;
                    if (!p.stall) {
                        mbar_expect_tx(&v_full[vs], p.kv_bytes);
                        for (int c = 0; c < nch; ++c)
                            tma_load_4d(sV + (size_t)vs * p.kv_bytes + c * BN * 128, &tmv, &v_full[vs],
                                        c * 64, w.h, j * BN, w.b);
                    }
                    if (++vs == p.nV) { vs = 0; vph ^= 1; }
                }
            }
        }
    } else if (warp == 1) {
        // ---------------- MMA issuer ----------------
        if (lane == 0) {
            // D fp32 (bit 4); A/B format at bits 7-9 / 10-12 (0 f16, 1 bf16);
            // bit 16: B is MN-major; N>>3 at bit 17, M>>4 at bit 24
            const uint32_t fmt = F16 ? 0u : 1u;
            const uint32_t idesc_s = (1u << 4) | (fmt << 7) | (fmt << 10) | ((uint32_t)(BN >> 3) << 17) |
                                     ((uint32_t)(BM >> 4) << 24);
            const uint32_t idesc_o = (1u << 4) | (fmt << 7) | (fmt << 10) | (1u << 16) |
                                     ((uint32_t)(p.D >> 3) << 17) | ((uint32_t)(BM >> 4) << 24);
            const uint32_t sq = smem_u32(sQ);
            int ks = 0, vs = 0;
            uint32_t kph = 0, vph = 0, qph = 0, G = 0;
            bool ok = true;
            // S_g = Q K^T for the key block in K stage ks
            auto issue_s = [&](uint32_t g) -> bool {
                if (!mbar_wait(&k_full[ks], kph, &s_abort, p.timeout_ns, flag)) return false;
                if (!mbar_wait(&s_free[g & 1], ((g >> 1) & 1) ^ 1, &s_abort, p.timeout_ns, flag))
                    return false;
                tc_fence_after();
                const uint32_t kb = smem_u32(sK + (size_t)ks * p.kv_bytes);
                const uint32_t d = tmem_base + (g & 1) * BN;
                for (int c = 0; c < nch; ++c) {
#pragma unroll
                    for (int kk = 0; kk < 4; ++kk)
                        umma<false>(d, sw128_desc(sq + c * BM * 128 + kk * 32),
                                    sw128_desc(kb + c * BN * 128 + kk * 32), idesc_s, (c | kk) != 0);
                }
                umma_commit(&k_empty[ks]);
                umma_commit(&s_full[g & 1]);
                if (++ks == p.nK) { ks = 0; kph ^= 1; }
                return true;
            };
            for (int u = blockIdx.x; ok && u < p.total_units; u += gridDim.x) {
                const Unit w = decode_unit(u, p);
                if (!(ok = mbar_wait(q_full, qph, &s_abort, p.timeout_ns, flag))) break;
                qph ^= 1;
                tc_fence_after();
                if (!(ok = issue_s(G))) break;
                for (int j = 0; j < w.nblk; ++j, ++G) {
                    if (j + 1 < w.nblk) {
                        if (!(ok = issue_s(G + 1))) break;
                    } else {
                        umma_commit(q_empty);  // every S of this unit is issued
                    }
                    const uint32_t pb = G & (uint32_t)(p.nP - 1);
                    if (!(ok = mbar_wait(&v_full[vs], vph, &s_abort, p.timeout_ns, flag))) break;
                    if (!(ok = mbar_wait(&p_full[pb], (G / p.nP) & 1, &s_abort, p.timeout_ns, flag)))
                        break;
                    tc_fence_after();
                    const uint32_t pa = smem_u32(sP + pb * PBYTES);
                    const uint32_t vb = smem_u32(sV + (size_t)vs * p.kv_bytes);
#pragma unroll
                    for (int kb = 0; kb < BN / 16; ++kb)
                        umma<false>(tmem_base + OCOL, sw128_desc(pa + (kb >> 2) * BM * 128 + (kb & 3) * 32),
                                    sw128_desc_mn(vb + kb * 16 * 128, BN * 128), idesc_o, (j | kb) != 0);
                    umma_commit(&v_empty[vs]);
                    umma_commit(&pv_done[G & 1]);
                    if (++vs == p.nV) { vs = 0; vph ^= 1; }
                }
            }
        }
    } else {
        // ---------------- softmax ----------------
        const int quarter = warp & 3;   // TMEM lanes this warp may access
        const int row = quarter * 32 + lane;
        const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
        const uint32_t s_col = tmem_base + lane_off;   // S buffer g&1 at column (g&1)*BN
        const uint32_t o_col = tmem_base + lane_off + OCOL;
        // all lanes of the warp take the same branch after every wait
        auto wait_all = [&](uint64_t* b, uint32_t parity) -> bool {
            const bool r = mbar_wait(b, parity, &s_abort, p.timeout_ns, flag);
            return __all_sync(0xffffffffu, r);
        };
        uint32_t G = 0;
        bool ok = true;
        for (int u = blockIdx.x; ok && u < p.total_units; u += gridDim.x) {
            const Unit w = decode_unit(u, p);
            const int64_t tq = (int64_t)w.qt * BM + row;
            const bool row_ok = tq < p.T_q;
            const uint32_t* brow = p.bits + ((int64_t)w.b * p.T_q + (row_ok ? tq : 0)) * p.words;
            float m_run = kNegInf, l = 0.f;
            uint4 mk = row_ok ? __ldg(reinterpret_cast<const uint4*>(brow)) : make_uint4(0, 0, 0, 0);
            for (int j = 0; j < w.nblk; ++j, ++G) {
                if (!(ok = wait_all(&s_full[G & 1], (G >> 1) & 1))) break;
                tc_fence_after();
                uint32_t s[128];
#pragma unroll
                for (int c = 0; c < 4; ++c) tmem_ld32(s_col + (G & 1) * BN + c * 32, s + c * 32);
#pragma unroll
                for (int c = 0; c < 4; ++c) tmem_wait_ld32(s + c * 32);
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&s_free[G & 1]);

                const uint32_t mw[4] = {mk.x, mk.y, mk.z, mk.w};
                if (row_ok && j + 1 < w.nblk)
                    mk = __ldg(reinterpret_cast<const uint4*>(brow) + j + 1);
                // dropped logits -> -inf; row max of the kept ones
                float mxp[8];
#pragma unroll
                for (int e = 0; e < 8; ++e) mxp[e] = kNegInf;
#pragma unroll
                for (int c = 0; c < 128; ++c) {
                    const float x = ((mw[c >> 5] >> (c & 31)) & 1u) ? __uint_as_float(s[c]) : kNegInf;
                    s[c] = __float_as_uint(x);
                    mxp[c & 7] = fmaxf(mxp[c & 7], x);
                }
                const float mx = fmaxf(fmaxf(fmaxf(mxp[0], mxp[1]), fmaxf(mxp[2], mxp[3])),
                                       fmaxf(fmaxf(mxp[4], mxp[5]), fmaxf(mxp[6], mxp[7])));
                const float m_new = fmaxf(m_run, mx * p.sl2);
                const bool need = m_new > m_run + 8.f;   // first kept logit, or growth > 2^8
                float alpha = 1.f;
                if (need) {
                    alpha = ex2(m_run - m_new);          // 0 while nothing was kept
                    m_run = m_new;
                    l *= alpha;
                }
                // the P buffer this block writes was read by PV_{G-nP}
                if (G >= (uint32_t)p.nP) {
                    const uint32_t g2 = G - p.nP;
                    if (!(ok = wait_all(&pv_done[g2 & 1], (g2 >> 1) & 1))) break;
                }
                if (j > 0 && __any_sync(0xffffffffu, need)) {
                    // rescale O in TMEM once PV_{G-1} has landed
                    if (p.nP == 2) {
                        const uint32_t g1 = G - 1;
                        if (!(ok = wait_all(&pv_done[g1 & 1], (g1 >> 1) & 1))) break;
                    }
                    tc_fence_after();
                    for (int c = 0; c < p.D / 32; ++c) {
                        uint32_t o[32];
                        tmem_ld32(o_col + c * 32, o);
                        tmem_wait_ld32(o);
#pragma unroll
                        for (int e = 0; e < 32; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * alpha);
                        tmem_st32(o_col + c * 32, o);
                    }
                    tmem_wait_st();
                }
                // P = exp2(x*sl2 - m) as 16-bit values, 128-byte swizzled K-major:
                // keys 64*cc + 8*i .. +7 of this row go to 16-byte slot i ^ (row & 7)
                const float mu = m_run == kNegInf ? 0.f : m_run;
                uint8_t* prow = sP + (G & (uint32_t)(p.nP - 1)) * PBYTES + row * 128;
                float lp[8];
#pragma unroll
                for (int e = 0; e < 8; ++e) lp[e] = 0.f;
#pragma unroll
                for (int cc = 0; cc < 2; ++cc) {
#pragma unroll
                    for (int i = 0; i < 8; ++i) {
                        float pv[8];
#pragma unroll
                        for (int e = 0; e < 8; ++e) {
                            pv[e] = ex2(fmaf(__uint_as_float(s[cc * 64 + i * 8 + e]), p.sl2, -mu));
                            lp[e] += pv[e];
                        }
                        uint4 pk;
                        pk.x = pack2(pv[0], pv[1], F16);
                        pk.y = pack2(pv[2], pv[3], F16);
                        pk.z = pack2(pv[4], pv[5], F16);
                        pk.w = pack2(pv[6], pv[7], F16);
                        *reinterpret_cast<uint4*>(prow + cc * BM * 128 + ((i ^ (row & 7)) << 4)) = pk;
                    }
                }
                l += ((lp[0] + lp[1]) + (lp[2] + lp[3])) + ((lp[4] + lp[5]) + (lp[6] + lp[7]));
                fence_async_smem();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&p_full[G & (uint32_t)(p.nP - 1)]);
            }
            if (!ok) break;
            // O / l after the unit's last PV
            {
                const uint32_t g1 = G - 1;
                if (!(ok = wait_all(&pv_done[g1 & 1], (g1 >> 1) & 1))) break;
            }
            tc_fence_after();
            const float inv = l > 0.f ? 1.f / l : 0.f;
            float* orow = p.O + (((int64_t)w.b * p.T_q + (row_ok ? tq : 0)) * p.HQ + w.h) * p.D;
            for (int c = 0; c < p.D / 32; ++c) {
                uint32_t o[32];
                tmem_ld32(o_col + c * 32, o);
                tmem_wait_ld32(o);
                if (row_ok) {
#pragma unroll
                    for (int e = 0; e < 32; e += 4)
                        *reinterpret_cast<float4*>(orow + c * 32 + e) =
                            make_float4(__uint_as_float(o[e]) * inv, __uint_as_float(o[e + 1]) * inv,
                                        __uint_as_float(o[e + 2]) * inv, __uint_as_float(o[e + 3]) * inv);
                }
            }
            tc_fence_before();
        }
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

// ---------------------------------------------------------------------------
// Two query tiles per work unit, ping-pong (the default kernel).
//
// A unit is (batch, head, query tiles 2m and 2m+1).  Both tiles are computed
// against the same K/V blocks, so every K/V block is loaded once for 256
// query rows, and two softmax warpgroups share the tensor core.  A softmax
// warpgroup frees its S columns as soon as it has read S_X(j) into registers
// (P goes to shared memory), so S_X(j+1) is computed while it still works on
// block j.  Issue order of the MMA warp: S_A(j), S_B(j), PV_A(j-1), PV_B(j-1).
//   warps 0..3   warp 0 TMA producer, warp 1 MMA issuer, warps 2-3 idle;
//                this warpgroup lowers its registers to 72 (setmaxnreg)
//   warps 4..7   softmax of tile A, warps 8..11 softmax of tile B; each
//                raises its registers to 216 and keeps its row of S_j (128
//                fp32 values) in registers
// TMEM (512 columns): S_A 0..127, O_A 128.., S_B 256..383, O_B 384..
// The launch needs 384 x 168 registers (the pool the two setmaxnreg steps
// redistribute: 128 x 72 + 256 x 216 = 384 x 168); the host checks the
// compiled register count before choosing this kernel.
constexpr int NT2 = 384;
constexpr uint32_t REG_LOW = 72, REG_HIGH = 216;
constexpr uint32_t REG_LAUNCH = 168;   // registers per thread the launch must have
static_assert(128 * REG_LOW + 256 * REG_HIGH == NT2 * REG_LAUNCH,
              "the setmaxnreg split must add up to the launch's register pool");

struct Unit2 {
    int b, h, qa, na, nb;   // tile A = qa, tile B = qa + 1 (nb = 0: no tile B)
};

__device__ __forceinline__ int tile_blocks(int qt, const AtParams& p) {
    int64_t tq_end = (int64_t)(qt + 1) * BM;
    if (tq_end > p.T_q) tq_end = p.T_q;
    int64_t nb = (p.q_row0 + tq_end - 1) / BN + 1;
    if (nb > p.nkb) nb = p.nkb;
    return (int)nb;
}

// unit index -> (batch, head, tile pair); the pairs with the most key blocks first
__device__ __forceinline__ Unit2 decode_unit2(int u, const AtParams& p) {
    Unit2 r;
    const int bh = p.B * p.HQ;
    const int npair = (p.n_qt + 1) >> 1;
    const int qr = u / bh, rem = u - qr * bh;
    const int m = npair - 1 - qr;
    r.b = rem / p.HQ;
    r.h = rem - r.b * p.HQ;
    r.qa = 2 * m;
    r.na = tile_blocks(r.qa, p);
    r.nb = r.qa + 1 < p.n_qt ? tile_blocks(r.qa + 1, p) : 0;
    return r;
}

template <bool F16>
__global__ void __launch_bounds__(NT2, 1)
    attn_tc2_kernel(const __grid_constant__ CUtensorMap tmq, const __grid_constant__ CUtensorMap tmk,
                    const __grid_constant__ CUtensorMap tmv, const AtParams p) {
    extern __shared__ uint8_t smem_raw[];
    __shared__ uint32_t tmem_slot;
    __shared__ int s_abort;
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                               ~uintptr_t(1023));
    // Q_A Q_B | K ring | V ring | P_A P_B | barriers (V is followed by P)
    uint8_t* sQ = smem;
    uint8_t* sK = sQ + 2 * (size_t)p.q_bytes;
    uint8_t* sV = sK + (size_t)p.nK * p.kv_bytes;
    uint8_t* sP = sV + (size_t)p.nV * p.kv_bytes;
    uint64_t* q_full = reinterpret_cast<uint64_t*>(sP + 2 * (size_t)PBYTES);
    uint64_t* q_empty = q_full + 1;
    uint64_t* k_full = q_empty + 1;
    uint64_t* k_empty = k_full + p.nK;
    uint64_t* v_full = k_empty + p.nK;
    uint64_t* v_empty = v_full + p.nV;
    uint64_t* s_full = v_empty + p.nV;   // [2] S_X(j) in TMEM
    uint64_t* s_free = s_full + 2;       // [2] softmax X has read S_X(j) into registers
    uint64_t* p_full = s_free + 2;       // [2] P_X(j) in shared memory
    uint64_t* pv_done = p_full + 2;      // [2] O_X += P_X(j) V(j) done

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nch = p.D / 64;
    int* flag = &g_attn_tc_timeout;

    if (threadIdx.x == 32) {
        s_abort = 0;
        // Q, K and V stages are released by both MMA issuers (one per tile)
        mbar_init(q_full, 1);
        mbar_init(q_empty, 2);
        for (int s = 0; s < p.nK; ++s) {
            mbar_init(&k_full[s], 1);
            mbar_init(&k_empty[s], 2);
        }
        for (int s = 0; s < p.nV; ++s) {
            mbar_init(&v_full[s], 1);
            mbar_init(&v_empty[s], 2);
        }
        for (int s = 0; s < 2; ++s) {
            mbar_init(&s_full[s], 1);
            mbar_init(&s_free[s], 4);
            mbar_init(&p_full[s], 4);
            mbar_init(&pv_done[s], 1);
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
    const int npair = (p.n_qt + 1) >> 1;
    const int total = npair * p.B * p.HQ;

    if (warp < 4) {
        asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(REG_LOW));
        if (warp == 0 && lane == 0) {
            // ---------------- TMA producer ----------------
            int ks = 0, vs = 0;
            uint32_t kph = 0, vph = 0, qph = 0;
            bool ok = true;
            for (int u = blockIdx.x; ok && u < total; u += gridDim.x) {
                const Unit2 w = decode_unit2(u, p);
                const int nblk = w.nb > w.na ? w.nb : w.na;
                if (!(ok = mbar_wait(q_empty, qph ^ 1, &s_abort, p.timeout_ns, flag))) break;
                qph ^= 1;
                if (!p.stall) {
                    mbar_expect_tx(q_full, p.q_bytes * (w.nb ? 2u : 1u));
                    for (int x = 0; x < (w.nb ? 2 : 1); ++x)
                        for (int c = 0; c < nch; ++c)
                            tma_load_4d(sQ + (size_t)x * p.q_bytes + c * BM * 128, &tmq, q_full, c * 64,
                                        w.h, (w.qa + x) * BM, w.b);
                }
                // K runs one block ahead of V: the MMA needs K(j+1) before V(j)
                auto load_k = [&](int jb) -> bool {
                    if (!mbar_wait(&k_empty[ks], kph ^ 1, &s_abort, p.timeout_ns, flag)) return false;
                    if (!p.stall) {
                        mbar_expect_tx(&k_full[ks], p.kv_bytes);
                        for (int c = 0; c < nch; ++c)
                            tma_load_4d(sK + (size_t)ks * p.kv_bytes + c * BN * 128, &tmk, &k_full[ks],
                                        c * 64, w.h, jb * BN, w.b);
                    }
                    if (++ks == p.nK) { ks = 0; kph ^= 1; }
                    return true;
                };
                if (!(ok = load_k(0))) break;
                for (int j = 0; j < nblk; ++j) {
                    if (j + 1 < nblk && !(ok = load_k(j + 1))) break;
                    if (!(ok = mbar_wait(&v_empty[vs], vph ^ 1, &s_abort, p.timeout_ns, flag))) break;
                    if (!p.stall) {
                        mbar_expect_tx(&v_full[vs], p.kv_bytes);
                        for (int c = 0; c < nch; ++c)
                            tma_load_4d(sV + (size_t)vs * p.kv_bytes + c * BN * 128, &tmv, &v_full[vs],
                                        c * 64, w.h, j * BN, w.b);
                    }
                    if (++vs == p.nV) { vs = 0; vph ^= 1; }
                }
            }
        } else if ((warp == 1 || warp == 2) && lane == 0) {
            // ---------------- MMA issuers: warp 1 for tile A, warp 2 for tile B ----------------
            // Each issuer waits only on its own tile's softmax, so one tile's PV
            // never queues behind the other tile's progress (tile B usually has
            // one more key block per unit).  Per key block j of its tile:
            // S(j+1) once the softmax has read S(j) out of TMEM, then PV(j) once
            // it has written P(j).  Blocks of the unit that only the other tile
            // uses are released without an MMA.
            const int x = warp - 1;
            const uint32_t fmt = F16 ? 0u : 1u;
            const uint32_t idesc_s = (1u << 4) | (fmt << 7) | (fmt << 10) | ((uint32_t)(BN >> 3) << 17) |
                                     ((uint32_t)(BM >> 4) << 24);
            const uint32_t idesc_o = (1u << 4) | (fmt << 7) | (fmt << 10) | (1u << 16) |
                                     ((uint32_t)(p.D >> 3) << 17) | ((uint32_t)(BM >> 4) << 24);
            const uint32_t qb = smem_u32(sQ + (size_t)x * p.q_bytes);
            const uint32_t s_tm = tmem_base + (uint32_t)x * 256u;
            const uint32_t o_tm = s_tm + 128u;
            const uint32_t pa = smem_u32(sP + (size_t)x * PBYTES);
            int ks = 0, vs = 0;
            uint32_t kph = 0, vph = 0, qph = 0, GS = 0, GP = 0;
            bool ok = true;
            auto k_next = [&]() { if (++ks == p.nK) { ks = 0; kph ^= 1; } };
            auto v_next = [&]() { if (++vs == p.nV) { vs = 0; vph ^= 1; } };
            // S = Q K^T into this tile's S columns, K from the current K stage
            auto issue_s = [&]() -> bool {
                if (!mbar_wait(&k_full[ks], kph, &s_abort, p.timeout_ns, flag)) return false;
                if (GS > 0 && !mbar_wait(&s_free[x], (GS - 1) & 1, &s_abort, p.timeout_ns, flag)) return false;
                tc_fence_after();
                const uint32_t kb = smem_u32(sK + (size_t)ks * p.kv_bytes);
                for (int c = 0; c < nch; ++c) {
#pragma unroll
                    for (int kk = 0; kk < 4; ++kk)
                        umma<false>(s_tm, sw128_desc(qb + c * BM * 128 + kk * 32),
                                    sw128_desc(kb + c * BN * 128 + kk * 32), idesc_s, (c | kk) != 0);
                }
                umma_commit(&s_full[x]);
                umma_commit(&k_empty[ks]);
                ++GS;
                k_next();
                return true;
            };
            // O (+)= P V, V from the current V stage
            auto issue_pv = [&](int j) -> bool {
                if (!mbar_wait(&v_full[vs], vph, &s_abort, p.timeout_ns, flag)) return false;
                if (!mbar_wait(&p_full[x], GP & 1, &s_abort, p.timeout_ns, flag)) return false;
                tc_fence_after();
                const uint32_t vb = smem_u32(sV + (size_t)vs * p.kv_bytes);
#pragma unroll
                for (int kb = 0; kb < BN / 16; ++kb)
                    umma<false>(o_tm, sw128_desc(pa + (kb >> 2) * BM * 128 + (kb & 3) * 32),
                                sw128_desc_mn(vb + kb * 16 * 128, BN * 128), idesc_o, (j | kb) != 0);
                umma_commit(&pv_done[x]);
                umma_commit(&v_empty[vs]);
                ++GP;
                v_next();
                return true;
            };
            // a K or V stage this tile does not use: wait for its fill, then release
            auto skip_stage = [&](uint64_t* full, uint64_t* empty, int st, uint32_t ph) -> bool {
                if (!mbar_wait(&full[st], ph, &s_abort, p.timeout_ns, flag)) return false;
                mbar_arrive(&empty[st]);
                return true;
            };
            for (int u = blockIdx.x; ok && u < total; u += gridDim.x) {
                const Unit2 w = decode_unit2(u, p);
                const int n = x == 0 ? w.na : w.nb;
                const int nblk = w.nb > w.na ? w.nb : w.na;
                if (!(ok = mbar_wait(q_full, qph, &s_abort, p.timeout_ns, flag))) break;
                qph ^= 1;
                if (n == 0) mbar_arrive(q_empty);
                else if (!(ok = issue_s())) break;
                if (n == 1) umma_commit(q_empty);
                for (int j = 0; ok && j < n; ++j) {
                    if (j + 1 < n) {
                        if (!(ok = issue_s())) break;
                        if (j + 2 == n) umma_commit(q_empty);   // this tile's last S was issued
                    }
                    if (!(ok = issue_pv(j))) break;
                }
                // blocks of this unit that only the other tile uses (K loads run one ahead of V)
                for (int j = n; ok && j < nblk; ++j) {
                    if (!(ok = skip_stage(k_full, k_empty, ks, kph))) break;
                    k_next();
                    if (!(ok = skip_stage(v_full, v_empty, vs, vph))) break;
                    v_next();
                }
            }
        }
    } else {
        asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(REG_HIGH));
        // ---------------- softmax: warpgroup x = 0 (tile A) or 1 (tile B) ----------------
        const int x = (warp >> 2) - 1;
        const int quarter = warp & 3;
        const int row = quarter * 32 + lane;
        const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
        const uint32_t s_col = tmem_base + lane_off + (uint32_t)x * 256u;
        const uint32_t o_col = s_col + 128u;
        uint8_t* prow_base = sP + (size_t)x * PBYTES + row * 128;
        auto wait_all = [&](uint64_t* b, uint32_t parity) -> bool {
            const bool r = mbar_wait(b, parity, &s_abort, p.timeout_ns, flag);
            return __all_sync(0xffffffffu, r);
        };
        uint32_t G = 0;
        bool ok = true;
        for (int u = blockIdx.x; ok && u < total; u += gridDim.x) {
            const Unit2 w = decode_unit2(u, p);
            const int nblk = x == 0 ? w.na : w.nb;
            if (nblk == 0) continue;
            const int qt = w.qa + x;
            const int64_t tq = (int64_t)qt * BM + row;
            const bool row_ok = tq < p.T_q;
            const uint32_t* brow = p.bits + ((int64_t)w.b * p.T_q + (row_ok ? tq : 0)) * p.words;
            float m_run = kNegInf, l = 0.f;
            uint4 mk = row_ok ? __ldg(reinterpret_cast<const uint4*>(brow)) : make_uint4(0, 0, 0, 0);
            for (int j = 0; j < nblk; ++j, ++G) {
                if (!(ok = wait_all(&s_full[x], G & 1))) break;
                tc_fence_after();
                uint32_t s[128];
#pragma unroll
                for (int c = 0; c < 4; ++c) tmem_ld32(s_col + c * 32, s + c * 32);
#pragma unroll
                for (int c = 0; c < 4; ++c) tmem_wait_ld32(s + c * 32);
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&s_free[x]);   // the MMA may write S_X(j+1)

                const uint32_t mw[4] = {mk.x, mk.y, mk.z, mk.w};
                if (row_ok && j + 1 < nblk) mk = __ldg(reinterpret_cast<const uint4*>(brow) + j + 1);
                // dropped logits -> -inf; row max of the kept ones (8 chains of 3-input max)
                float mxp[8];
#pragma unroll
                for (int e = 0; e < 8; ++e) mxp[e] = kNegInf;
#pragma unroll
                for (int c = 0; c < 128; c += 2) {
                    const float v0 = ((mw[c >> 5] >> (c & 31)) & 1u) ? __uint_as_float(s[c]) : kNegInf;
                    const float v1 =
                        ((mw[c >> 5] >> ((c + 1) & 31)) & 1u) ? __uint_as_float(s[c + 1]) : kNegInf;
                    s[c] = __float_as_uint(v0);
                    s[c + 1] = __float_as_uint(v1);
                    mxp[(c >> 1) & 7] = fmax3(mxp[(c >> 1) & 7], v0, v1);
                }
                const float mx = fmax3(fmax3(mxp[0], mxp[1], mxp[2]), fmax3(mxp[3], mxp[4], mxp[5]),
                                       fmaxf(mxp[6], mxp[7]));
                const float m_new = fmaxf(m_run, mx * p.sl2);
                const bool need = m_new > m_run + 8.f;
                float alpha = 1.f;
                if (need) {
                    alpha = ex2(m_run - m_new);
                    m_run = m_new;
                    l *= alpha;
                }
                // P_X's buffer and O_X: PV_X(j-1) must have landed
                if (j > 0 && !(ok = wait_all(&pv_done[x], (G - 1) & 1))) break;
                // P = 2^(x*sl2 - m): the exponent in fp32 (packed FMA), 2^ in fp32
                // on the MUFU, rounded to the 16-bit input type for the PV product;
                // l sums the fp32 values (packed adds).  16-byte slot i of the
                // 128-byte swizzled row holds keys 64*cc + 8*i .. +7.
                const float mu = m_run == kNegInf ? 0.f : m_run;
                const float2 sl2v = make_float2(p.sl2, p.sl2), nmu = make_float2(-mu, -mu);
                uint64_t lp[4] = {0ull, 0ull, 0ull, 0ull};   // packed fp32 pairs
#pragma unroll
                for (int cc = 0; cc < 2; ++cc) {
#pragma unroll
                    for (int i = 0; i < 8; ++i) {
                        uint32_t pk[4];
#pragma unroll
                        for (int e = 0; e < 4; ++e) {
                            const int c = cc * 64 + i * 8 + 2 * e;
                            const float2 xx =
                                fma2(make_float2(__uint_as_float(s[c]), __uint_as_float(s[c + 1])), sl2v, nmu);
                            pk[e] = ex2_pair_sum<F16>(xx.x, xx.y, lp[e]);
                        }
                        *reinterpret_cast<uint4*>(prow_base + cc * BM * 128 + ((i ^ (row & 7)) << 4)) =
                            make_uint4(pk[0], pk[1], pk[2], pk[3]);
                    }
                }
                {
                    float f[8];
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        f[2 * e] = __uint_as_float((uint32_t)lp[e]);
                        f[2 * e + 1] = __uint_as_float((uint32_t)(lp[e] >> 32));
                    }
                    l += ((f[0] + f[1]) + (f[2] + f[3])) + ((f[4] + f[5]) + (f[6] + f[7]));
                }
                // rescale O_X (after the row's S values are dead); PV_X(j) is
                // issued only after p_full, so it sees the rescaled O
                if (j > 0 && __any_sync(0xffffffffu, need)) {
                    tc_fence_after();
                    for (int c = 0; c < p.D / 32; ++c) {
                        uint32_t o[32];
                        tmem_ld32(o_col + c * 32, o);
                        tmem_wait_ld32(o);
#pragma unroll
                        for (int e = 0; e < 32; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * alpha);
                        tmem_st32(o_col + c * 32, o);
                    }
                    tmem_wait_st();
                }
                fence_async_smem();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&p_full[x]);
            }
            if (!ok) break;
            if (!(ok = wait_all(&pv_done[x], (G - 1) & 1))) break;
            tc_fence_after();
            const float inv = l > 0.f ? 1.f / l : 0.f;
            float* orow = p.O + (((int64_t)w.b * p.T_q + (row_ok ? tq : 0)) * p.HQ + w.h) * p.D;
            for (int c = 0; c < p.D / 32; ++c) {
                uint32_t o[32];
                tmem_ld32(o_col + c * 32, o);
                tmem_wait_ld32(o);
                if (row_ok && p.o_vec8) {
                    // 32-byte stores: whole sectors of each of the warp's 32 rows
#pragma unroll
                    for (int e = 0; e < 32; e += 8)
                        asm volatile("st.global.v8.f32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"l"(orow + c * 32 + e),
                                     "f"(__uint_as_float(o[e]) * inv), "f"(__uint_as_float(o[e + 1]) * inv),
                                     "f"(__uint_as_float(o[e + 2]) * inv), "f"(__uint_as_float(o[e + 3]) * inv),
                                     "f"(__uint_as_float(o[e + 4]) * inv), "f"(__uint_as_float(o[e + 5]) * inv),
                                     "f"(__uint_as_float(o[e + 6]) * inv), "f"(__uint_as_float(o[e + 7]) * inv)
                                     : "memory");
                } else if (row_ok) {
#pragma unroll
                    for (int e = 0; e < 32; e += 4)
                        *reinterpret_cast<float4*>(orow + c * 32 + e) =
                            make_float4(__uint_as_float(o[e]) * inv, __uint_as_float(o[e + 1]) * inv,
                                        __uint_as_float(o[e + 2]) * inv, __uint_as_float(o[e + 3]) * inv);
                }
            }
            tc_fence_before();
        }
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

// Kept-set bitmap: bit (s & 31) of word s/32 of query row r is set iff
// s <= q_row0 + r % T_q and scores[r, s] >= thr[r].  One CTA per query row;
// each warp turns 32 consecutive scores into one word with a ballot.  Words
// past the causal end (up to `words`) are written as zero.
__global__ void __launch_bounds__(256) kept_bitmap_kernel(const float* __restrict__ scores,
                                                          const float* __restrict__ thr,
                                                          uint32_t* __restrict__ bits, int64_t T_q,
                                                          int64_t T_k, int64_t q_row0, int64_t words) {
    const int64_t row = blockIdx.x;
    int64_t last = q_row0 + row % T_q;   // last causal key
    if (last > T_k - 1) last = T_k - 1;
    const float th = thr[row];
    const float* srow = scores + row * T_k;
    uint32_t* brow = bits + row * words;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
#pragma unroll 4
    for (int64_t wd = warp; wd < words; wd += 8) {
        const int64_t s = wd * 32 + lane;
        const bool keep = s <= last && __ldg(srow + s) >= th;
        const uint32_t m = __ballot_sync(0xffffffffu, keep);
        if (lane == 0) brow[wd] = m;
    }
}

}  // namespace

int64_t bitmap_words(int64_t T_k) { return ((T_k + BN - 1) / BN) * (BN / 32); }

int kept_bitmap(const float* scores, const float* thr, uint32_t* bits, int64_t B, int64_t T_q,
                int64_t T_k, int64_t q_row0, int64_t words, cudaStream_t stream) {
    if (!scores || !thr || !bits) return fail(DSA_ERR_INVALID, "kept_bitmap: null pointer");
    if (B < 0 || T_q < 0 || T_k < 1 || q_row0 < 0)
        return fail(DSA_ERR_INVALID, "kept_bitmap: bad sizes");
    if (words < bitmap_words(T_k) || (words & 3))
        return fail(DSA_ERR_INVALID, "kept_bitmap: words_per_row must be a multiple of 4 and >= "
                                     "dsa_bitmap_words(T_k)");
    const int64_t rows = B * T_q;
    if (rows == 0) return DSA_OK;
    if (rows > INT32_MAX) return fail(DSA_ERR_INVALID, "kept_bitmap: too many rows");
    kept_bitmap_kernel<<<(unsigned)rows, 256, 0, stream>>>(scores, thr, bits, T_q, T_k, q_row0, words);
    return check_launch("kept_bitmap_kernel");
}

// Synchronises `stream`, reads and clears the timeout flag of this device.
int attn_tc_take_timeout(cudaStream_t stream) {
    if (cudaStreamSynchronize(stream) != cudaSuccess) return -1;
    int flag = 0;
    if (cudaMemcpyFromSymbol(&flag, g_attn_tc_timeout, sizeof(int)) != cudaSuccess) return -1;
    if (flag) {
        const int zero = 0;
        if (cudaMemcpyToSymbol(g_attn_tc_timeout, &zero, sizeof(int)) != cudaSuccess) return -1;
    }
    return flag ? 1 : 0;
}

bool attn_tc_supported(int64_t HQ, int64_t DQ, int64_t DV, int dtype) {
    return (dtype == DSA_BF16 || dtype == DSA_F16) && DQ == DV && (DQ == 64 || DQ == 128) &&
           HQ >= 1 && HQ <= 65535;
}

// Returns -100 when the shape is outside this kernel's limits (the caller
// uses the gather kernel instead).
int attn_tc(const uint32_t* bits, int64_t words, const void* Q, const void* K, const void* V,
            float* O, int64_t B, int64_t T_q, int64_t T_k, int64_t q_row0, int64_t HQ, int64_t D,
            float scale, int dtype, cudaStream_t stream) {
    if (!attn_tc_supported(HQ, D, D, dtype)) return -100;
    if (!aligned16(Q) || !aligned16(K) || !aligned16(V) || !aligned16(O) || !aligned16(bits))
        return -100;
    AtParams p;
    p.O = O;
    p.bits = bits;
    p.words = words;
    p.T_q = T_q;
    p.T_k = T_k;
    p.q_row0 = q_row0;
    p.B = (int)B;
    p.HQ = (int)HQ;
    p.D = (int)D;
    p.n_qt = (int)((T_q + BM - 1) / BM);
    p.nkb = (int)((T_k + BN - 1) / BN);
    const int64_t units = (int64_t)p.n_qt * B * HQ;
    if (units > INT32_MAX || T_q > INT32_MAX || T_k > INT32_MAX) return -100;
    p.total_units = (int)units;
    p.q_bytes = (uint32_t)(BM * D * 2);
    p.kv_bytes = (uint32_t)(BN * D * 2);
    p.sl2 = scale * 1.4426950408889634f;
    // DSA_TEST_ATTN_STALL=1: test hook for the timeout path (no loads are
    // issued, every wait runs out after 20 ms); never set in normal use
    p.stall = getenv("DSA_TEST_ATTN_STALL") ? 1 : 0;
    p.timeout_ns = p.stall ? 20000000ull : 2000000000ull;
    p.o_vec8 = (reinterpret_cast<uintptr_t>(O) & 31u) == 0 ? 1 : 0;
    if (units == 0) return DSA_OK;

    int dev = 0, optin = 0;
    if (cudaGetDevice(&dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev) != cudaSuccess)
        return fail(DSA_ERR_CUDA, "attn_tc: cannot query shared memory limits");
    // The two-tile kernel redistributes a launch pool of exactly 384 x 168
    // registers; it runs only when the compiled kernel asks for that many.
    auto kern2 = dtype == DSA_F16 ? attn_tc2_kernel<true> : attn_tc2_kernel<false>;
    auto kern1 = dtype == DSA_F16 ? attn_tc_kernel<true> : attn_tc_kernel<false>;
    cudaFuncAttributes fa2, fa1;
    if (cudaFuncGetAttributes(&fa2, kern2) != cudaSuccess || cudaFuncGetAttributes(&fa1, kern1) != cudaSuccess)
        return fail(DSA_ERR_CUDA, "attn_tc: cannot query kernel attributes");
    bool two = fa2.numRegs == (int)REG_LAUNCH && !getenv("DSA_ATTN_TC_ONE_TILE");
    size_t smem = 0;
    if (two) {
        // Q_A Q_B, P_A P_B, then as many K and V stages as fit (K first)
        const size_t avail = (size_t)optin - fa2.sharedSizeBytes - 1024 - 256;
        const size_t fixed = 2 * (size_t)p.q_bytes + 2 * (size_t)PBYTES;
        const int n = avail > fixed ? (int)((avail - fixed) / p.kv_bytes) : 0;
        if (n < 3) {
            two = false;
        } else {
            p.nV = n / 2 > 4 ? 4 : n / 2;
            p.nK = n - p.nV > 4 ? 4 : n - p.nV;
            // DSA_ATTN_KV=<nK>,<nV>: ring depths for tuning (each >= 1, sum <= n)
            if (const char* kv = getenv("DSA_ATTN_KV")) {
                int a = 0, b = 0;
                if (sscanf(kv, "%d,%d", &a, &b) == 2 && a >= 1 && b >= 1 && a + b <= n && a <= 4 && b <= 4) {
                    p.nK = a;
                    p.nV = b;
                }
            }
            p.nP = 2;
            smem = 1024 + 256 + fixed + (size_t)(p.nK + p.nV) * p.kv_bytes;
        }
    }
    if (!two) {
        // one tile per unit: K and V stages of equal depth (2..4), two P buffers when they fit
        const size_t avail = (size_t)optin - fa1.sharedSizeBytes - 1024 - 256;
        p.nP = 2;
        size_t rest = avail - p.q_bytes - 2 * (size_t)PBYTES;
        int n = (int)(rest / (2 * (size_t)p.kv_bytes));
        if (n < 2) {
            p.nP = 1;
            rest = avail - p.q_bytes - PBYTES;
            n = (int)(rest / (2 * (size_t)p.kv_bytes));
        }
        if (n < 2) return -100;
        if (n > 4) n = 4;
        p.nK = p.nV = n;
        smem = 1024 + 256 + p.q_bytes + (size_t)(p.nK + p.nV) * p.kv_bytes + (size_t)p.nP * PBYTES;
    }

    const CUtensorMapDataType dt = dtype == DSA_F16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16
                                                    : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
    CUtensorMap tmq, tmk, tmv;
    const cuuint32_t box[4] = {64, 1, 128, 1};
    {
        const cuuint64_t dims[4] = {(cuuint64_t)D, (cuuint64_t)HQ, (cuuint64_t)T_q, (cuuint64_t)B};
        const cuuint64_t str[3] = {(cuuint64_t)D * 2, (cuuint64_t)(HQ * D * 2),
                                   (cuuint64_t)(T_q * HQ * D * 2)};
        int rc = encode_map(&tmq, Q, 4, dims, str, box, "attn_tc: Q", dt);
        if (rc) return rc;
    }
    {
        const cuuint64_t dims[4] = {(cuuint64_t)D, (cuuint64_t)HQ, (cuuint64_t)T_k, (cuuint64_t)B};
        const cuuint64_t str[3] = {(cuuint64_t)D * 2, (cuuint64_t)(HQ * D * 2),
                                   (cuuint64_t)(T_k * HQ * D * 2)};
        int rc = encode_map(&tmk, K, 4, dims, str, box, "attn_tc: K", dt);
        if (rc) return rc;
        rc = encode_map(&tmv, V, 4, dims, str, box, "attn_tc: V", dt);
        if (rc) return rc;
    }
    auto kern = two ? kern2 : kern1;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
        return fail(DSA_ERR_CUDA, "attn_tc: cannot set dynamic shared memory size");
    const int64_t work = two ? (int64_t)((p.n_qt + 1) / 2) * B * HQ : p.total_units;
    int grid = num_sms();
    if (grid > work) grid = (int)work;
    kern<<<grid, two ? NT2 : NTHREADS, smem, stream>>>(tmq, tmk, tmv, p);
    return check_launch(two ? "attn_tc2_kernel" : "attn_tc_kernel");
}

}  // namespace dsa
