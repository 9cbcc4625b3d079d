// Row arithmetic shared by the prologue (K1: the appended row of each decode
// step) and the prefill hand-off (mla_rows.cu: rows written into pages in bulk):
// the cache row of one token is RMSNorm(c) | RoPE(k_pe) of its raw kv_a, with
// the rounding points of reference_decode.py:51-65, 120-134, 230-237.
#pragma once

#include "mla_common.cuh"

namespace mla {

// DeepseekV2 RoPE on 64 values x[0..64): interleave-transpose, then rotate_half
// (reference_decode.py:120-134). For pair j < 32:
//   out[j]    = x[2j]*cos[j]       - x[2j+1]*sin[j]
//   out[32+j] = x[2j+1]*cos[32+j]  + x[2j]*sin[32+j]
// Products and the sum are rounded separately, as NumPy evaluates
// `x * cos + rotate_half(x) * sin`.
// rope_pair with the pair's table entries already loaded: c_lo = cos[j], s_lo = sin[j],
// c_hi = cos[32 + j], s_hi = sin[32 + j].
__device__ __forceinline__ void rope_pair_r(float x_even, float x_odd, float c_lo, float s_lo, float c_hi, float s_hi,
                                            float& lo, float& hi) {
    lo = __fadd_rn(__fmul_rn(x_even, c_lo), -__fmul_rn(x_odd, s_lo));
    hi = __fadd_rn(__fmul_rn(x_odd, c_hi), __fmul_rn(x_even, s_hi));
}
__device__ __forceinline__ void rope_pair(float x_even, float x_odd, const float* cs, const float* sn, int j,
                                          float& lo, float& hi) {
    rope_pair_r(x_even, x_odd, cs[j], sn[j], cs[32 + j], sn[32 + j], lo, hi);
}

// The raw values one lane of kv_post needs: c[16 lane, 16 lane + 16) of the kv_a
// row, gamma over the same columns and k_pe pair `lane`. Loaded apart from the
// arithmetic, so that a caller can issue these loads with its other independent
// ones (they do not depend on the row's position).
struct KvPostIn {
    float x[16];
    __align__(16) __nv_bfloat16 gw[16];
    float kp0, kp1;
};

// gam = nullptr: the caller fills in.gw itself.
__device__ __forceinline__ void kv_post_load(const __nv_bfloat16* src, const __nv_bfloat16* gam, int lane,
                                             KvPostIn& in) {
    {
        const uint4* s4 = reinterpret_cast<const uint4*>(src) + 2 * lane;
        uint4 v[2];
        if ((reinterpret_cast<uintptr_t>(src) & 15) == 0) {
            v[0] = s4[0]; v[1] = s4[1];
            const __nv_bfloat162* h2 = reinterpret_cast<const __nv_bfloat162*>(v);
#pragma unroll
            for (int k = 0; k < 8; ++k) { in.x[2 * k] = __low2float(h2[k]); in.x[2 * k + 1] = __high2float(h2[k]); }
        } else {
#pragma unroll
            for (int k = 0; k < 16; ++k) in.x[k] = __bfloat162float(src[16 * lane + k]);
        }
    }
    if (gam == nullptr) {
    } else if ((reinterpret_cast<uintptr_t>(gam) & 15) == 0) {
        reinterpret_cast<uint4*>(in.gw)[0] = reinterpret_cast<const uint4*>(gam)[2 * lane];
        reinterpret_cast<uint4*>(in.gw)[1] = reinterpret_cast<const uint4*>(gam)[2 * lane + 1];
    } else {
#pragma unroll
        for (int k = 0; k < 16; ++k) in.gw[k] = gam[16 * lane + k];
    }
    const __nv_bfloat16* kp = src + kLora + 2 * lane;
    in.kp0 = __bfloat162float(kp[0]);
    in.kp1 = __bfloat162float(kp[1]);
}

// One warp: the cache row of the loaded raw kv_a values at a RoPE position whose
// table entries for this lane's pair are c_lo = cos[lane], s_lo = sin[lane],
// c_hi = cos[32 + lane], s_hi = sin[32 + lane]. Lane owns c[16 lane, 16 lane + 16)
// (outc) and RoPE pair `lane` of k_pe (lo -> column 512 + lane, hi -> 544 + lane).
__device__ __forceinline__ void kv_post_finish_r(const KvPostIn& in, float eps, float c_lo, float s_lo, float c_hi,
                                                 float s_hi, int lane, __nv_bfloat16 (&outc)[16], float& lo,
                                                 float& hi) {
    // kv_post (reference_decode.py:60-65): var = mean(x^2); y = x * (1 / sqrt(var + eps));
    // row = bf16(bf16(y) * weight). Lane owns c[16*lane, 16*lane+16).
    float ss = 0.f;
#pragma unroll
    for (int k = 0; k < 16; ++k) ss = __fadd_rn(ss, __fmul_rn(in.x[k], in.x[k]));
#pragma unroll
    for (int o = 16; o; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    const float var = __fdiv_rn(ss, (float)kLora);
    const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(var, eps)));
#pragma unroll
    for (int k = 0; k < 16; ++k) {
        const float y = bf16_round(__fmul_rn(in.x[k], inv));
        outc[k] = __float2bfloat16_rn(__fmul_rn(y, __bfloat162float(in.gw[k])));
    }
    rope_pair_r(in.kp0, in.kp1, c_lo, s_lo, c_hi, s_hi, lo, hi);
}

// The same with the position's tables cs / sn in memory.
__device__ __forceinline__ void kv_post_finish(const KvPostIn& in, float eps, const float* cs, const float* sn,
                                               int lane, __nv_bfloat16 (&outc)[16], float& lo, float& hi) {
    kv_post_finish_r(in, eps, cs[lane], sn[lane], cs[32 + lane], sn[32 + lane], lane, outc, lo, hi);
}

// kv_post_load + kv_post_finish, for callers with nothing to overlap.
__device__ __forceinline__ void kv_post_compute(const __nv_bfloat16* src, const __nv_bfloat16* gam, float eps,
                                                const float* cs, const float* sn, int lane,
                                                __nv_bfloat16 (&outc)[16], float& lo, float& hi) {
    KvPostIn in;
    kv_post_load(src, gam, lane, in);
    kv_post_finish(in, eps, cs, sn, lane, outc, lo, hi);
}

// Store a row computed by kv_post_compute; dst is 16-byte aligned.
__device__ __forceinline__ void kv_post_store(__nv_bfloat16* dst, const __nv_bfloat16 (&outc)[16], float lo, float hi,
                                              int lane) {
    reinterpret_cast<uint4*>(dst)[2 * lane] = reinterpret_cast<const uint4*>(outc)[0];
    reinterpret_cast<uint4*>(dst)[2 * lane + 1] = reinterpret_cast<const uint4*>(outc)[1];
    dst[kLora + lane] = __float2bfloat16_rn(lo);
    dst[kLora + 32 + lane] = __float2bfloat16_rn(hi);
}

}  // namespace mla
