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
//               each CTA loads its own tiles) through two mbarrier rings
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
    int64_t row_bstep;    // batch b's query rows start at q_row0 + b*row_bstep
    int kshared, vshared; // K / V have batch stride 0: every batch reads batch 0
    int B, HQ, D;
    int n_qt, nkb, total_units;
    int nK, nV, nP;
    uint32_t q_bytes, kv_bytes;
    float sl2;            // scale * log2(e)
    int stall;            // test hook: the producer issues no loads, so every wait times out
    int o_vec8;           // O 32-byte aligned: 256-bit output stores
    const float* vscale;  // V was converted to fp16 as V / *vscale (power of two); O is scaled back
    const uint32_t* summ; // per (batch, query tile): one bit per key block holding any kept key, or null
    int sw;               // summary words per query tile
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
    int64_t nb = (p.q_row0 + r.b * p.row_bstep + tq_end - 1) / BN + 1;
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

template <bool F16, bool PV16>
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
                                        c * 64, w.h, j * BN, p.kshared ? 0 : w.b);
                    }
                    if (++ks == p.nK) { ks = 0; kph ^= 1; }
                    if (!(ok = mbar_wait(&v_empty[vs], vph ^ 1, &s_abort, p.timeout_ns, flag))) break;
                    if (!p.stall) {
                        mbar_expect_tx(&v_full[vs], p.kv_bytes);
                        for (int c = 0; c < nch; ++c)
                            tma_load_4d(sV + (size_t)vs * p.kv_bytes + c * BN * 128, &tmv, &v_full[vs],
                                        c * 64, w.h, j * BN, p.vshared ? 0 : w.b);
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
            const uint32_t fmt_o = PV16 ? 0u : 1u;   // P and V: fp16 or bf16
            const uint32_t idesc_o = (1u << 4) | (fmt_o << 7) | (fmt_o << 10) | (1u << 16) |
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
                        pk.x = pack2(pv[0], pv[1], PV16);
                        pk.y = pack2(pv[2], pv[3], PV16);
                        pk.z = pack2(pv[4], pv[5], PV16);
                        pk.w = pack2(pv[6], pv[7], PV16);
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
            // an empty kept set (a NaN threshold) gives NaN, as the reference's
            // softmax over all -inf logits does
            const float inv = (l > 0.f ? 1.f / l : __uint_as_float(0x7fc00000u)) *
                              (p.vscale ? __ldg(p.vscale) : 1.f);
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

__device__ __forceinline__ int tile_blocks(int qt, int b, const AtParams& p) {
    int64_t tq_end = (int64_t)(qt + 1) * BM;
    if (tq_end > p.T_q) tq_end = p.T_q;
    int64_t nb = (p.q_row0 + b * p.row_bstep + tq_end - 1) / BN + 1;
    if (nb > p.nkb) nb = p.nkb;
    return (int)nb;
}

// unit index -> (batch, head, tile pair); the pairs with the most key blocks first
// Units in decreasing size (key blocks grow with the tiles' absolute rows):
// with one row offset for every batch, by pair from the last, then batch and
// head; with row blocks that do not overlap (row_bstep >= the block's rows),
// by batch from the last, then pair from the last, then head.
__device__ __forceinline__ Unit2 decode_unit2(int u, const AtParams& p) {
    Unit2 r;
    const int bh = p.B * p.HQ;
    const int npair = (p.n_qt + 1) >> 1;
    int m;
    if (p.row_bstep >= p.T_q && p.B > 1) {
        const int e = u / p.HQ;
        r.h = u - e * p.HQ;
        r.b = p.B - 1 - e / npair;
        m = npair - 1 - (e - (e / npair) * npair);
    } else {
        const int qr = u / bh, rem = u - qr * bh;
        m = npair - 1 - qr;
        r.b = rem / p.HQ;
        r.h = rem - r.b * p.HQ;
    }
    r.qa = 2 * m;
    r.na = tile_blocks(r.qa, r.b, p);
    r.nb = r.qa + 1 < p.n_qt ? tile_blocks(r.qa + 1, r.b, p) : 0;
    DSA_CHECK(r.b < p.B && r.qa < p.n_qt && r.na <= p.nkb, DBG_TILE);   // flagged only
    return r;
}

// The k-th unit of this CTA: units are dealt to the CTAs in rounds, forward
// in even rounds and backward in odd ones ("snake"), so with units in
// decreasing size a CTA that drew a large unit early draws a small one next.
// Returns a value >= total when this CTA has no unit in round k.
__device__ __forceinline__ int snake_unit(int k) {
    const int G = (int)gridDim.x;
    return k * G + ((k & 1) ? G - 1 - (int)blockIdx.x : (int)blockIdx.x);
}

// Whether key block j holds a kept key of query tile qt (always, without a summary).
__device__ __forceinline__ bool block_used(const AtParams& p, int b, int qt, int j) {
    return !p.summ || ((__ldg(p.summ + ((int64_t)b * p.n_qt + qt) * p.sw + (j >> 5)) >> (j & 31)) & 1u);
}
// Whether every key block 0..n-1 of query tile qt is used (then the walks
// over a unit's blocks take every block without reading the summary again).
__device__ __forceinline__ bool tile_full(const AtParams& p, int b, int qt, int n) {
    if (!p.summ) return true;
    const uint32_t* w = p.summ + ((int64_t)b * p.n_qt + qt) * p.sw;
    for (int i = 0; i * 32 < n; ++i) {
        const int left = n - i * 32;
        const uint32_t need = left >= 32 ? 0xffffffffu : ((1u << left) - 1u);
        if ((__ldg(w + i) & need) != need) return false;
    }
    return true;
}

template <bool F16, bool PV16>
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
            for (int kr = 0; ok && kr * (int)gridDim.x < total; ++kr) {
                const int u = snake_unit(kr);
                if (u >= total) continue;
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
                                        c * 64, w.h, jb * BN, p.kshared ? 0 : w.b);
                    }
                    if (++ks == p.nK) { ks = 0; kph ^= 1; }
                    return true;
                };
                // the unit's key blocks: those either tile uses (all causal ones
                // without a summary); K runs one used block ahead of V
                const bool dense = tile_full(p, w.b, w.qa, w.na) && (w.nb == 0 || tile_full(p, w.b, w.qa + 1, w.nb));
                auto next_used = [&](int j) {
                    if (dense) return j + 1;
                    do { ++j; } while (j < nblk && !((j < w.na && block_used(p, w.b, w.qa, j)) ||
                                                     (j < w.nb && block_used(p, w.b, w.qa + 1, j))));
                    return j;
                };
                int j = next_used(-1);
                if (j < nblk && !(ok = load_k(j))) break;
                for (; j < nblk;) {
                    const int jn = next_used(j);
                    if (jn < nblk && !(ok = load_k(jn))) break;
                    if (!(ok = mbar_wait(&v_empty[vs], vph ^ 1, &s_abort, p.timeout_ns, flag))) break;
                    if (!p.stall) {
                        mbar_expect_tx(&v_full[vs], p.kv_bytes);
                        for (int c = 0; c < nch; ++c)
                            tma_load_4d(sV + (size_t)vs * p.kv_bytes + c * BN * 128, &tmv, &v_full[vs],
                                        c * 64, w.h, j * BN, p.vshared ? 0 : w.b);
                    }
                    if (++vs == p.nV) { vs = 0; vph ^= 1; }
                    j = jn;
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
            const uint32_t fmt_o = PV16 ? 0u : 1u;   // P and V: fp16 or bf16
            const uint32_t idesc_o = (1u << 4) | (fmt_o << 7) | (fmt_o << 10) | (1u << 16) |
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
            auto issue_pv = [&](bool first) -> bool {
                if (!mbar_wait(&v_full[vs], vph, &s_abort, p.timeout_ns, flag)) return false;
                if (!mbar_wait(&p_full[x], GP & 1, &s_abort, p.timeout_ns, flag)) return false;
                tc_fence_after();
                const uint32_t vb = smem_u32(sV + (size_t)vs * p.kv_bytes);
#pragma unroll
                for (int kb = 0; kb < BN / 16; ++kb)
                    umma<false>(o_tm, sw128_desc(pa + (kb >> 2) * BM * 128 + (kb & 3) * 32),
                                sw128_desc_mn(vb + kb * 16 * 128, BN * 128), idesc_o, !first || kb != 0);
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
            for (int kr = 0; ok && kr * (int)gridDim.x < total; ++kr) {
                const int u = snake_unit(kr);
                if (u >= total) continue;
                const Unit2 w = decode_unit2(u, p);
                const int n = x == 0 ? w.na : w.nb;
                const int nblk = w.nb > w.na ? w.nb : w.na;
                if (!(ok = mbar_wait(q_full, qph, &s_abort, p.timeout_ns, flag))) break;
                qph ^= 1;
                // The stages arrive in the producer's order K(u0), then K(u_i+1)
                // before V(u_i) over the unit's used blocks u_i; they are taken in
                // that order.  A block of this tile gets its S (on K) and PV (on
                // V) MMA; a block only the other tile uses is released.
                const bool fullA = tile_full(p, w.b, w.qa, w.na);
                const bool fullB = w.nb == 0 || tile_full(p, w.b, w.qa + 1, w.nb);
                const bool full_x = x == 0 ? fullA : fullB;
                auto mine = [&](int j) { return j < n && (full_x || block_used(p, w.b, w.qa + x, j)); };
                auto next_used = [&](int j) {
                    if (fullA && fullB) return j + 1;
                    do { ++j; } while (j < nblk && !((j < w.na && block_used(p, w.b, w.qa, j)) ||
                                                     (j < w.nb && block_used(p, w.b, w.qa + 1, j))));
                    return j;
                };
                int last = -1;   // this tile's last block: Q is free once its S is issued
                for (int j = n - 1; j >= 0 && last < 0; --j)
                    if (mine(j)) last = j;
                if (last < 0) mbar_arrive(q_empty);
                bool first = true;
                auto take_k = [&](int j) -> bool {
                    if (mine(j)) {
                        if (!issue_s()) return false;
                        if (j == last) umma_commit(q_empty);
                        return true;
                    }
                    if (!skip_stage(k_full, k_empty, ks, kph)) return false;
                    k_next();
                    return true;
                };
                auto take_v = [&](int j) -> bool {
                    if (mine(j)) {
                        if (!issue_pv(first)) return false;
                        first = false;
                        return true;
                    }
                    if (!skip_stage(v_full, v_empty, vs, vph)) return false;
                    v_next();
                    return true;
                };
                int j = next_used(-1);
                if (j < nblk && !(ok = take_k(j))) break;
                while (j < nblk) {
                    const int jn = next_used(j);
                    if (jn < nblk && !(ok = take_k(jn))) break;
                    if (!(ok = take_v(j))) break;
                    j = jn;
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
        for (int kr = 0; ok && kr * (int)gridDim.x < total; ++kr) {
            const int u = snake_unit(kr);
            if (u >= total) continue;
            const Unit2 w = decode_unit2(u, p);
            const int nblk = x == 0 ? w.na : w.nb;
            if (nblk == 0) continue;
            const int qt = w.qa + x;
            const int64_t tq = (int64_t)qt * BM + row;
            const bool row_ok = tq < p.T_q;
            const uint32_t* brow = p.bits + ((int64_t)w.b * p.T_q + (row_ok ? tq : 0)) * p.words;
            float m_run = kNegInf, l = 0.f;
            // this tile's key blocks (those holding a kept key of the tile)
            const bool full = tile_full(p, w.b, qt, nblk);
            auto next_mine = [&](int j) {
                if (full) return j + 1;
                do { ++j; } while (j < nblk && !block_used(p, w.b, qt, j));
                return j;
            };
            int j = next_mine(-1);
            uint4 mk = row_ok && j < nblk ? __ldg(reinterpret_cast<const uint4*>(brow) + j) : make_uint4(0, 0, 0, 0);
            int jj = 0;   // ordinal of block j among the tile's blocks
            for (; j < nblk; ++jj, ++G) {
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
                const int jn = next_mine(j);
                if (row_ok && jn < nblk) mk = __ldg(reinterpret_cast<const uint4*>(brow) + jn);
                j = jn;
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
                if (jj > 0 && !(ok = wait_all(&pv_done[x], (G - 1) & 1))) break;
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
                            pk[e] = ex2_pair_sum<PV16>(xx.x, xx.y, lp[e]);
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
                if (jj > 0 && __any_sync(0xffffffffu, need)) {
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
            if (jj == 0) {
                // no key block of this tile holds a kept key: every row's kept set
                // is empty (NaN thresholds), and so is its output (NaN, as the
                // reference's softmax over all -inf logits)
                float* orow = p.O + (((int64_t)w.b * p.T_q + (row_ok ? tq : 0)) * p.HQ + w.h) * p.D;
                if (row_ok)
                    for (int c = 0; c < p.D; ++c) orow[c] = __uint_as_float(0x7fc00000u);
                continue;
            }
            if (!(ok = wait_all(&pv_done[x], (G - 1) & 1))) break;
            tc_fence_after();
            // an empty kept set (a NaN threshold) gives NaN, as the reference's
            // softmax over all -inf logits does
            const float inv = (l > 0.f ? 1.f / l : __uint_as_float(0x7fc00000u)) *
                              (p.vscale ? __ldg(p.vscale) : 1.f);
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
// s <= q_row0 + (r / T_q)*row_bstep + r % T_q and scores[r, s] >= thr[r].  One CTA per query row;
// each warp turns 32 consecutive scores into one word with a ballot.  Words
// past the causal end (up to `words`) are written as zero.
__global__ void __launch_bounds__(256) kept_bitmap_kernel(const float* __restrict__ scores,
                                                          const float* __restrict__ thr,
                                                          uint32_t* __restrict__ bits, int64_t T_q,
                                                          int64_t T_k, int64_t q_row0, int64_t words,
                                                          int64_t row_bstep) {
    const int64_t row = blockIdx.x;
    int64_t last = q_row0 + (row / T_q) * row_bstep + row % T_q;   // last causal key
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

// ---- V in fp16 for the P.V product ------------------------------------------
// With bf16 inputs the softmax weights P would enter the P.V MMA as bf16 (an
// 8-bit significand: up to 2^-9 relative error per weight).  One MMA takes one
// operand type, so P in fp16 (11 bits, 8x finer) needs V in fp16 too: V is
// copied once per call as fp16(V / s), s a power of two with max|V| / s <=
// 2^15 (exact scaling; every bf16 value in that range is exact in fp16), and
// the output is multiplied back by s.  Non-finite V keeps s = 1.

// max |V| as float bits (non-negative floats order like their bit patterns;
// NaN's bits exceed +inf's).  V rows of D elements at b*sb + t*sr + h*sh.
__global__ void __launch_bounds__(256) v_absmax_kernel(const __nv_bfloat16* __restrict__ V, int64_t T_k,
                                                       int HQ, int D, int64_t sb, int64_t sr, int64_t sh,
                                                       int64_t chunks, uint32_t* __restrict__ amax) {
    const int cpr = D / 8;   // 16-byte chunks per row
    uint32_t m = 0;
    for (int64_t c = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; c < chunks;
         c += (int64_t)gridDim.x * blockDim.x) {
        const int64_t row = c / cpr;
        const int off = (int)(c - row * cpr) * 8;
        const int h = (int)(row % HQ);
        const int64_t bt = row / HQ;
        const int64_t t = bt % T_k, b = bt / T_k;
        const uint4 v = ldg16(V + b * sb + t * sr + h * sh + off);
        const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const uint32_t lo = (w[i] << 16) & 0x7fffffffu, hi = w[i] & 0x7fff0000u;
            m = max(m, max(lo, hi));
        }
    }
    m = __reduce_max_sync(0xffffffffu, m);
    if ((threadIdx.x & 31) == 0 && m) atomicMax(amax, m);
}

__global__ void __launch_bounds__(256) v_to_f16_kernel(const __nv_bfloat16* __restrict__ V, int64_t T_k,
                                                       int HQ, int D, int64_t sb, int64_t sr, int64_t sh,
                                                       int64_t chunks, const uint32_t* __restrict__ amax,
                                                       __half* __restrict__ out, float* __restrict__ scale) {
    const float a = __uint_as_float(*amax);
    float s = 1.f;
    if (a <= 3.4028234663852886e38f)           // finite: smallest power of two with a / s <= 2^15
        while (a > 32768.f * s) s *= 2.f;
    const float inv = 1.f / s;                 // a power of two: exact
    if (blockIdx.x == 0 && threadIdx.x == 0) *scale = s;
    const int cpr = D / 8;
    for (int64_t c = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; c < chunks;
         c += (int64_t)gridDim.x * blockDim.x) {
        const int64_t row = c / cpr;
        const int off = (int)(c - row * cpr) * 8;
        const int h = (int)(row % HQ);
        const int64_t bt = row / HQ;
        const int64_t t = bt % T_k, b = bt / T_k;
        const uint4 v = ldg16(V + b * sb + t * sr + h * sh + off);
        const uint32_t w[4] = {v.x, v.y, v.z, v.w};
        uint32_t o[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const __half2 hv = __floats2half2_rn(__uint_as_float(w[i] << 16) * inv,
                                                 __uint_as_float(w[i] & 0xffff0000u) * inv);
            o[i] = *reinterpret_cast<const uint32_t*>(&hv);
        }
        *reinterpret_cast<uint4*>(out + row * D + off) = make_uint4(o[0], o[1], o[2], o[3]);
    }
}

// Block summary of the kept-set bitmap: bit j of word (b*n_qt + qt)*sw + j/32
// is set iff key block j holds a kept key of some row of query tile qt.  One
// CTA per (query tile, batch); thread t ORs key block t (t + 256, ...) over
// the tile's rows, each row's block read as one 16-byte load.
__global__ void __launch_bounds__(256) block_summary_kernel(const uint32_t* __restrict__ bits, int64_t words,
                                                            int64_t T_q, int n_qt, int nkb, int sw,
                                                            uint32_t* __restrict__ summ) {
    const int qt = blockIdx.x, b = blockIdx.y;
    const int64_t r0 = (int64_t)qt * BM;
    const int nr = (int)(T_q - r0 < BM ? T_q - r0 : BM);
    const uint32_t* tile = bits + ((int64_t)b * T_q + r0) * words;
    uint32_t* out = summ + ((int64_t)b * n_qt + qt) * sw;
    for (int j0 = 0; j0 < sw * 32; j0 += blockDim.x) {
        const int j = j0 + threadIdx.x;
        uint32_t any = 0;
        if (j < nkb) {
            const uint4* col = reinterpret_cast<const uint4*>(tile) + j;
            const int64_t stride = words / 4;
#pragma unroll 8
            for (int r = 0; r < nr; ++r) {
                const uint4 v = __ldg(col + r * stride);
                any |= v.x | v.y | v.z | v.w;
            }
        }
        const uint32_t m = __ballot_sync(0xffffffffu, any != 0);
        if ((threadIdx.x & 31) == 0 && j < sw * 32) out[j >> 5] = m;
    }
}

}  // namespace

// Workspace of dsa_sparse_attn_bitmap_ex: a 256-byte header (max |V|, the V
// scale), the block summary [B, n_qt, ceil(nkb/32)] uint32 (256-byte
// aligned), and for bf16 inputs the fp16 copy of V [B, T_k, HQ, D].
static size_t summ_bytes(int64_t B, int64_t T_q, int64_t T_k) {
    const int64_t n_qt = (T_q + BM - 1) / BM, nkb = (T_k + BN - 1) / BN;
    return (((size_t)B * n_qt * ((nkb + 31) / 32) * 4) + 255) & ~size_t(255);
}
size_t attn_ws_bytes(int64_t B, int64_t T_q, int64_t T_k, int64_t HQ, int64_t D, int dtype) {
    return 256 + summ_bytes(B, T_q, T_k) +
           (dtype == DSA_BF16 ? (size_t)B * (size_t)T_k * (size_t)HQ * (size_t)D * 2 : 0);
}

int64_t bitmap_words(int64_t T_k) { return ((T_k + BN - 1) / BN) * (BN / 32); }

int kept_bitmap(const float* scores, const float* thr, uint32_t* bits, int64_t B, int64_t T_q,
                int64_t T_k, int64_t q_row0, int64_t words, int64_t row_bstep, cudaStream_t stream) {
    if (!scores || !thr || !bits) return fail(DSA_ERR_INVALID, "kept_bitmap: null pointer");
    if (B < 0 || T_q < 0 || T_k < 1 || q_row0 < 0)
        return fail(DSA_ERR_INVALID, "kept_bitmap: bad sizes");
    if (words < bitmap_words(T_k) || (words & 3))
        return fail(DSA_ERR_INVALID, "kept_bitmap: words_per_row must be a multiple of 4 and >= "
                                     "dsa_bitmap_words(T_k)");
    const int64_t rows = B * T_q;
    if (rows == 0) return DSA_OK;
    if (rows > INT32_MAX) return fail(DSA_ERR_INVALID, "kept_bitmap: too many rows");
    kept_bitmap_kernel<<<(unsigned)rows, 256, 0, stream>>>(scores, thr, bits, T_q, T_k, q_row0, words,
                                                           row_bstep);
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
            float scale, int dtype, const dsa_layout& L, void* ws, size_t ws_bytes, cudaStream_t stream) {
    if (!attn_tc_supported(HQ, D, D, dtype)) return -100;
    if (!aligned16(Q) || !aligned16(K) || !aligned16(V) || !aligned16(O) || !aligned16(bits))
        return -100;
    // tensor-map strides: positive multiples of 16 bytes; a K or V batch
    // stride of 0 is read as one shared batch
    for (int i = 1; i < 3; ++i)
        if (!tma_stride_ok(L.Q[i], 2) || !tma_stride_ok(L.K[i], 2) || !tma_stride_ok(L.V[i], 2)) return -100;
    if (B > 1 && (!tma_stride_ok(L.Q[0], 2) || (L.K[0] != 0 && !tma_stride_ok(L.K[0], 2)) ||
                  (L.V[0] != 0 && !tma_stride_ok(L.V[0], 2))))
        return -100;
    AtParams p;
    p.O = O;
    p.bits = bits;
    p.words = words;
    p.T_q = T_q;
    p.T_k = T_k;
    p.q_row0 = q_row0;
    p.row_bstep = L.row_bstep;
    p.kshared = (B > 1 && L.K[0] == 0) ? 1 : 0;
    p.vshared = (B > 1 && L.V[0] == 0) ? 1 : 0;
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
    p.vscale = nullptr;
    p.summ = nullptr;
    p.sw = (p.nkb + 31) / 32;
    // with a workspace: the block summary (key blocks no row of a query tile
    // keeps are skipped), and for bf16 inputs the fp16 copy of V (P.V in fp16,
    // see v_to_f16_kernel)
    const int64_t B_v = p.vshared ? 1 : B;
    const size_t sbytes = summ_bytes(B, T_q, T_k);
    const bool have_ws = ws && (reinterpret_cast<uintptr_t>(ws) & 255u) == 0 && ws_bytes >= 256 + sbytes;
    const bool v16 = dtype == DSA_BF16 && have_ws &&
                     ws_bytes >= 256 + sbytes + (size_t)B_v * T_k * HQ * D * 2;
    const bool pv16 = dtype == DSA_F16 || v16;
    // DSA_ATTN_NO_SKIP=1: process every causal key block (cross-check of the skipping)
    const bool skip = have_ws && !getenv("DSA_ATTN_NO_SKIP");
    if (units == 0) return DSA_OK;

    int dev = 0, optin = 0;
    if (cudaGetDevice(&dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev) != cudaSuccess)
        return fail(DSA_ERR_CUDA, "attn_tc: cannot query shared memory limits");
    // The two-tile kernel redistributes a launch pool of exactly 384 x 168
    // registers; it runs only when the compiled kernel asks for that many.
    auto kern2 = dtype == DSA_F16 ? attn_tc2_kernel<true, true>
                 : pv16          ? attn_tc2_kernel<false, true>
                                 : attn_tc2_kernel<false, false>;
    auto kern1 = dtype == DSA_F16 ? attn_tc_kernel<true, true>
                 : pv16          ? attn_tc_kernel<false, true>
                                 : attn_tc_kernel<false, false>;
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
        const cuuint64_t str[3] = {(cuuint64_t)L.Q[2] * 2, (cuuint64_t)L.Q[1] * 2,
                                   (cuuint64_t)(B > 1 ? L.Q[0] : L.Q[1] * T_q) * 2};
        int rc = encode_map(&tmq, Q, 4, dims, str, box, "attn_tc: Q", dt);
        if (rc) return rc;
    }
    const void* Vsrc = V;
    int64_t vst[3] = {L.V[0], L.V[1], L.V[2]};
    if (v16) {
        // the fp16 copy of V (contiguous [B_v, T_k, HQ, D]) and its scale
        uint32_t* amax = static_cast<uint32_t*>(ws);
        float* vscale = reinterpret_cast<float*>(static_cast<char*>(ws) + 4);
        __half* V16 = reinterpret_cast<__half*>(static_cast<char*>(ws) + 256 + sbytes);
        const int64_t chunks = B_v * T_k * HQ * (D / 8);
        int grid = num_sms() * 8;
        if ((int64_t)grid * 256 > chunks) grid = (int)((chunks + 255) / 256);
        if (cudaMemsetAsync(amax, 0, sizeof(uint32_t), stream) != cudaSuccess)
            return fail(DSA_ERR_CUDA, "attn_tc: cudaMemsetAsync failed");
        const __nv_bfloat16* Vb = static_cast<const __nv_bfloat16*>(V);
        v_absmax_kernel<<<grid, 256, 0, stream>>>(Vb, T_k, (int)HQ, (int)D, L.V[0], L.V[1], L.V[2], chunks, amax);
        int rc = check_launch("v_absmax_kernel");
        if (rc) return rc;
        v_to_f16_kernel<<<grid, 256, 0, stream>>>(Vb, T_k, (int)HQ, (int)D, L.V[0], L.V[1], L.V[2], chunks,
                                                  amax, V16, vscale);
        if ((rc = check_launch("v_to_f16_kernel"))) return rc;
        p.vscale = vscale;
        Vsrc = V16;
        vst[2] = D;
        vst[1] = HQ * D;
        vst[0] = p.vshared ? 0 : T_k * HQ * D;
    }
    {
        // one map per tensor; a shared batch is a batch dimension of 1
        const int64_t* st[2] = {L.K, vst};
        const void* base[2] = {K, Vsrc};
        const int shared[2] = {p.kshared, p.vshared};
        const CUtensorMapDataType dts[2] = {dt, pv16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : dt};
        CUtensorMap* m[2] = {&tmk, &tmv};
        for (int x = 0; x < 2; ++x) {
            const cuuint64_t dims[4] = {(cuuint64_t)D, (cuuint64_t)HQ, (cuuint64_t)T_k,
                                        (cuuint64_t)(shared[x] ? 1 : B)};
            const cuuint64_t str[3] = {(cuuint64_t)st[x][2] * 2, (cuuint64_t)st[x][1] * 2,
                                       (cuuint64_t)(B > 1 && !shared[x] ? st[x][0] : st[x][1] * T_k) * 2};
            int rc = encode_map(m[x], base[x], 4, dims, str, box, x ? "attn_tc: V" : "attn_tc: K", dts[x]);
            if (rc) return rc;
        }
    }
    if (skip && two) {
        uint32_t* summ = reinterpret_cast<uint32_t*>(static_cast<char*>(ws) + 256);
        block_summary_kernel<<<dim3((unsigned)p.n_qt, (unsigned)B), 256, 0, stream>>>(bits, words, T_q, p.n_qt,
                                                                                   p.nkb, p.sw, summ);
        const int rc = check_launch("block_summary_kernel");
        if (rc) return rc;
        p.summ = summ;
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

DSA_DEBUG_FLAGS_READER(attn_tc)

}  // namespace dsa
