// Shared helpers of the DSA B200 kernels: status reporting, element loads,
// float <-> radix-key mapping.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <string>

#include "../../include/dsa_b200.h"

namespace dsa {

// ---- host-side status ----------------------------------------------------
void set_error(const std::string& msg);
void clear_error();
int fail(int code, const std::string& msg);
int check_launch(const char* what);
int num_sms();

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// The caller's layout, or the contiguous one when it passed none.
inline dsa_layout layout_or_contiguous(const dsa_layout* l, int64_t T_q, int64_t T_k, int64_t HI,
                                       int64_t DI, int64_t HQ, int64_t DQ, int64_t DV) {
    if (l) return *l;
    dsa_layout c;
    c.q[2] = DI; c.q[1] = HI * DI; c.q[0] = T_q * HI * DI;
    c.k[1] = DI; c.k[0] = T_k * DI;
    c.w[1] = HI; c.w[0] = T_q * HI;
    c.Q[2] = DQ; c.Q[1] = HQ * DQ; c.Q[0] = T_q * HQ * DQ;
    c.K[2] = DQ; c.K[1] = HQ * DQ; c.K[0] = T_k * HQ * DQ;
    c.V[2] = DV; c.V[1] = HQ * DV; c.V[0] = T_k * HQ * DV;
    c.row_bstep = 0;
    return c;
}
// A byte stride a TMA tensor map accepts: a positive multiple of 16 below 2^40.
inline bool tma_stride_ok(int64_t elems, int64_t elt) {
    const int64_t b = elems * elt;
    return b > 0 && (b & 15) == 0 && b < (int64_t(1) << 40);
}
inline size_t dtype_size(int dt) { return dt == DSA_F32 ? 4 : dt == DSA_FP8_E4M3 ? 1 : 2; }
// dtypes of the indexer inputs (q, k); the attention inputs exclude FP8
inline bool dtype_ok(int dt) {
    return dt == DSA_F32 || dt == DSA_BF16 || dt == DSA_F16 || dt == DSA_FP8_E4M3;
}

// ---- device helpers --------------------------------------------------------
template <typename T> struct Elem;
template <> struct Elem<float> {
    static __device__ __forceinline__ float to_f(float x) { return x; }
};
template <> struct Elem<__nv_bfloat16> {
    static __device__ __forceinline__ float to_f(__nv_bfloat16 x) { return __bfloat162float(x); }
};
template <> struct Elem<__half> {
    static __device__ __forceinline__ float to_f(__half x) { return __half2float(x); }
};
template <> struct Elem<__nv_fp8_e4m3> {
    static __device__ __forceinline__ float to_f(__nv_fp8_e4m3 x) { return float(x); }
};

// 16 bytes of T -> 16/sizeof(T) floats.
template <typename T>
__device__ __forceinline__ void unpack16(const uint4& v, float* out);
template <>
__device__ __forceinline__ void unpack16<float>(const uint4& v, float* out) {
    out[0] = __uint_as_float(v.x); out[1] = __uint_as_float(v.y);
    out[2] = __uint_as_float(v.z); out[3] = __uint_as_float(v.w);
}
template <>
__device__ __forceinline__ void unpack16<__nv_bfloat16>(const uint4& v, float* out) {
    // bf16 -> fp32 is a 16-bit left shift of the bit pattern.
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        out[2 * i] = __uint_as_float(w[i] << 16);
        out[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
    }
}
template <>
__device__ __forceinline__ void unpack16<__half>(const uint4& v, float* out) {
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        __half2 h = *reinterpret_cast<const __half2*>(&w[i]);
        float2 f = __half22float2(h);
        out[2 * i] = f.x;
        out[2 * i + 1] = f.y;
    }
}

// Order-preserving map float -> uint32 (larger float -> larger key), with
// the value order of torch.topk: -0.0 is folded onto +0.0 (key equality is
// float ==), and every NaN, whatever its sign and payload, maps to the one
// largest key KEY_NAN (torch.topk ranks NaN above +inf).  A NaN counts
// towards the k largest but is never kept: the selection rule is
// score >= threshold, which is false for NaN (see kept_key).
constexpr uint32_t KEY_NAN = 0xffffffffu;
__device__ __forceinline__ uint32_t f2key(float x) {
    // negative: ~b, positive: b | sign; then -0 (key 0x7fffffff) -> +0's key
    const uint32_t b = __float_as_uint(x);
    const uint32_t k = b ^ ((uint32_t)((int32_t)b >> 31) | 0x80000000u);
    const uint32_t k0 = k == 0x7fffffffu ? 0x80000000u : k;
    return (b & 0x7fffffffu) > 0x7f800000u ? KEY_NAN : k0;
}
// f2key without the NaN canonicalisation (NaNs keep distinct keys at both
// ends: -NaN below -inf, +NaN above +inf).  Equal to f2key on every non-NaN
// value; hot sweeps use it where a row without keys in the edge bins (which
// hold every NaN) is then known to hold no NaN.
__device__ __forceinline__ uint32_t f2key_raw(float x) {
    const uint32_t b = __float_as_uint(x);
    const uint32_t k = b ^ ((uint32_t)((int32_t)b >> 31) | 0x80000000u);
    return k == 0x7fffffffu ? 0x80000000u : k;
}
// Whether a score of key `key` is kept under threshold key `thr_key`
// (score >= thr as floats: NaN scores are never kept, a NaN threshold keeps nothing).
__device__ __forceinline__ bool kept_key(uint32_t key, uint32_t thr_key) {
    return key >= thr_key && key != KEY_NAN;
}
__device__ __forceinline__ float key2f(uint32_t k) {
    uint32_t b = (k & 0x80000000u) ? (k & 0x7fffffffu) : ~k;
    return __uint_as_float(b);
}

// ---- the checked build (-DDSA_DEBUG_CHECKS, libdsa_b200_checked.so) ----------
// DSA_CHECK(cond, bit) is true in the normal build.  In the checked build a
// false cond ORs `bit` into this file's device flag word instead of letting
// the guarded access happen (the caller skips it); dsa_debug_status() reads
// and clears every file's word.  No trap, no fault.
enum DebugBit : unsigned {
    DBG_LIST_KEY = 1u,      // a kept-index list entry outside 0 <= s <= t (stage 3 list form)
    DBG_CAND_OVERFLOW = 2u, // a top-K candidate past the candidate buffer
    DBG_TILE = 4u,          // a decoded tile / unit outside the launch's shape
    DBG_WORD = 8u,          // a bitmap word past the row's words
};
#ifdef DSA_DEBUG_CHECKS
static __device__ unsigned int g_dsa_debug_flags;   // one word per .cu file (no relocatable device code)
__device__ __forceinline__ bool dsa_check_fail(unsigned bit) {
    atomicOr(&g_dsa_debug_flags, bit);
    return false;
}
#define DSA_CHECK(cond, bit) ((cond) ? true : ::dsa::dsa_check_fail(bit))
// host: read and clear this file's flag word (0 on error)
static inline unsigned take_debug_flags_here() {
    unsigned f = 0, z = 0;
    if (cudaMemcpyFromSymbol(&f, g_dsa_debug_flags, sizeof f) != cudaSuccess) return 0;
    if (f) cudaMemcpyToSymbol(g_dsa_debug_flags, &z, sizeof z);
    return f;
}
#else
#define DSA_CHECK(cond, bit) true
static inline unsigned take_debug_flags_here() { return 0; }
#endif
// Each kernel file exports its flag reader under its own name.
#define DSA_DEBUG_FLAGS_READER(name) \
    unsigned debug_flags_##name() { return take_debug_flags_here(); }

__device__ __forceinline__ uint4 ldg16(const void* p) {
    return __ldg(reinterpret_cast<const uint4*>(p));
}

}  // namespace dsa
