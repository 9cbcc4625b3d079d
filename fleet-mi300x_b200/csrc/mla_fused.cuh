// The one-kernel step (MLA_FLAG_FUSED_STEP): for one request, the split-KV kernel
// also runs the prologue before its loop and the merge + W_UV after it, so a
// decode step is one launch instead of three dependent ones (K1, K2, K3). What a
// one-request step pays is mostly fixed latency: each kernel boundary costs a
// grid drain and a release, and K2's first tiles wait for K1. Here every CTA
// requests its first half pages at once, while the first 65 CTAs do K1's work:
//   * CTAs [0, 64): the absorb, one (head h, quarter j of the latent) slice each:
//     q_c[h][128j, 128j+128) = q_nope[h] W_UK[h][:, 128j : 128j+128] (fp32 sums of
//     exact bf16 products, rounded to bf16), reference_decode.py:250;
//   * CTA 64: q_pe RoPE and the appended cache row (K1's per-request warp,
//     reference_decode.py:231-237), unless the call stores no row.
// Each signals `ready`; every CTA waits for all 65 before its score MMAs and before
// requesting the half page that holds the new row. After the loop, every CTA
// signals `done`, and CTA (h, j) < 128 folds all partials of head h over its 64
// latent columns [64j, 64j+64) (weights 2^(m_c - M), M the max over partials, in
// plan order), divides by L and multiplies by W_UV[h][:, 64j : 64j+64]: a partial
// of y[h] = W_UV[h] o_c[h] over 64 latent columns (fp32 o_c times bf16 weights,
// exact products). The last of the 8 slices of a head adds the 8 partials in
// slice order and writes R(out) (or this shard's y, m, L: shard_out, or the
// peer-exchange lines that K4 combines).
//
// Ordering: counters in the workspace's sync region, written by atomics after a
// __threadfence(); readers poll with ld.acquire, bounded by the same 1.5 s limit as
// every other wait (then MLA_DEV_TIMEOUT, `abort` set, the others stop waiting).
// A CTA waits only for CTAs of its own grid, so the whole grid must be resident at
// once: the host launches it only where one CTA per SM fits for the whole grid, and
// the kernel lets the next kernel on the stream launch (griddepcontrol) only after
// its own CTAs have passed the prologue wait, so a dependent kernel never takes the
// SM of a CTA of this one that has not started yet. The new row is written with
// generic stores and read by TMA (the async proxy): both sides fence the proxies.
// The last CTA to finish zeroes the counters for the next step.
#pragma once

#include "mla_common.cuh"
#include "mla_rowops.cuh"

namespace mla {
namespace fused {

constexpr int kAbsorbCtas = kHeads * 4;        // (head, quarter of the latent) slices
constexpr int kRowCta = kAbsorbCtas;           // q_pe RoPE and the new row
constexpr int kPrologueCtas = kAbsorbCtas + 1;
constexpr int kMergeCtas = kHeads * kFyParts;  // (head, 64 latent columns)
constexpr int kMinCtas = kMergeCtas;           // the grid holds every merge slice (and the prologue)
constexpr int kMaxParts = 512;                 // partials of one request the merge can weigh (plan CTAs)
static_assert(kMinCtas >= kPrologueCtas, "the grid must hold the prologue CTAs");

__device__ __forceinline__ uint32_t ld_acquire(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void fence_proxy_async_global() {
    asm volatile("fence.proxy.async.global;" ::: "memory");
}

// One thread: wait until *ctr >= target. False if the step aborted or the wait ran
// out (then MLA_DEV_TIMEOUT is recorded and the step aborted).
__device__ inline bool wait_count(FusedSync* s, const uint32_t* ctr, uint32_t target, const ErrSink& err) {
    if (ld_acquire(ctr) >= target) return true;
    const uint64_t t0 = globaltimer_ns();
    for (uint32_t i = 1;; ++i) {
        __nanosleep(32);
        if (ld_acquire(ctr) >= target) return true;
        if ((i & 15) == 0) {
            if (*reinterpret_cast<volatile uint32_t*>(&s->abort)) return false;
            if (globaltimer_ns() - t0 > kWaitLimitNs) {
                record_error(err, MLA_DEV_TIMEOUT);
                atomicExch(&s->abort, 1u);
                return false;
            }
        }
    }
}

// All threads of the CTA: this CTA's global writes (and, for TMA readers, the new
// row) are visible before thread 0 counts it in *ctr.
__device__ inline void signal(uint32_t* ctr) {
    __threadfence();
    fence_proxy_async_global();
    __syncthreads();
    if (threadIdx.x == 0) atomicAdd(ctr, 1u);
}

// The absorb slice's W_UK values, loaded before the wait on the previous kernel (a
// weight: no kernel writes it) and before this CTA requests any cache tile, so that
// they are not queued behind the step's first tiles. Thread t holds the 8 latent
// columns 128j + 8 (t & 15) + [0, 8) of the 8 rows d = 8 (t >> 4) + [0, 8) of W_UK[h]
// (kv_b rows 256h + d), as loaded (nothing consumes them before the wait). The step's
// q_nope row is prefetched into L2 (the point of coherence, so a later write by the
// previous kernel is still seen).
struct AbsorbPre {
    uint4 w[8];
};
__device__ inline void absorb_pre(const MlaDecodeParams& p, int slice, AbsorbPre& a) {
    const int h = slice >> 2, j = slice & 3, cg = threadIdx.x & 15, rg = threadIdx.x >> 4;
    const uint4* w = reinterpret_cast<const uint4*>(reinterpret_cast<const __nv_bfloat16*>(p.kv_b) +
                                                    (int64_t)(h * kKvbHead + 8 * rg) * kLora + 128 * j + 8 * cg);
#pragma unroll
    for (int i = 0; i < 8; ++i) a.w[i] = w[(int64_t)i * (kLora / 8)];
    if (threadIdx.x == 0) {
        const char* q = reinterpret_cast<const char*>(p.q) + (int64_t)h * kQHead * 2;
        asm volatile("prefetch.global.L2 [%0];" ::"l"(q) : "memory");
        asm volatile("prefetch.global.L2 [%0];" ::"l"(q + 128) : "memory");
    }
}

// After the wait: the slice's 128 values of q_c, rounded to bf16 into qa. scratch:
// 128 + 16 * 128 floats of shared memory. Every thread of the CTA calls it.
__device__ inline void absorb_finish(const MlaDecodeParams& p, int slice, const AbsorbPre& a, __nv_bfloat16* qa,
                                     float* scratch) {
    const int h = slice >> 2, j = slice & 3, t = threadIdx.x, cg = t & 15, rg = t >> 4;
    float* qs = scratch;         // q_nope[h], 128 values
    float* red = scratch + 128;  // [16 row groups][128 columns]
    if (t < kNope)
        qs[t] = __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p.q)[(int64_t)h * kQHead + t]);
    __syncthreads();
    float acc[8];
#pragma unroll
    for (int c = 0; c < 8; ++c) acc[c] = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const float qv = qs[8 * rg + i];
        const __nv_bfloat162* w2 = reinterpret_cast<const __nv_bfloat162*>(&a.w[i]);
#pragma unroll
        for (int c = 0; c < 4; ++c) {
            acc[2 * c] = fmaf(qv, __low2float(w2[c]), acc[2 * c]);
            acc[2 * c + 1] = fmaf(qv, __high2float(w2[c]), acc[2 * c + 1]);
        }
    }
#pragma unroll
    for (int c = 0; c < 8; ++c) red[rg * 128 + 8 * cg + c] = acc[c];
    __syncthreads();
    if (t < 128) {
        float v = 0.f;
#pragma unroll
        for (int r = 0; r < 16; ++r) v += red[r * 128 + t];
        qa[(int64_t)h * kRow + 128 * j + t] = __float2bfloat16_rn(v);
    }
}

// The merge slice's W_UV values, loaded before its wait (a weight): thread t owns
// row v = t >> 1 of W_UV[h] (kv_b row 256h + 128 + v) over the 32 latent columns
// [64j + 32 (t & 1), +32).
struct UvPre {
    uint4 w[4];
};
__device__ inline void uv_pre(const MlaDecodeParams& p, int item, UvPre& u) {
    const int h = item / kFyParts, j = item % kFyParts, t = threadIdx.x;
    const uint4* w = reinterpret_cast<const uint4*>(reinterpret_cast<const __nv_bfloat16*>(p.kv_b) +
                                                    (int64_t)(h * kKvbHead + kNope + (t >> 1)) * kLora + 64 * j +
                                                    32 * (t & 1));
#pragma unroll
    for (int k = 0; k < 4; ++k) u.w[k] = w[k];
}

// Block-wide reductions over 256 threads in a fixed order (warp butterflies, then the
// eight warp results in warp order), so every slice of a head gets the same bits.
__device__ inline float block_max(float v, float* sc) {
#pragma unroll
    for (int o = 16; o; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    __syncthreads();
    if ((threadIdx.x & 31) == 0) sc[threadIdx.x >> 5] = v;
    __syncthreads();
    float m = sc[0];
#pragma unroll
    for (int w = 1; w < 8; ++w) m = fmaxf(m, sc[w]);
    return m;
}
__device__ inline float block_sum(float v, float* sc) {
#pragma unroll
    for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    __syncthreads();
    if ((threadIdx.x & 31) == 0) sc[threadIdx.x >> 5] = v;
    __syncthreads();
    float s = sc[0];
#pragma unroll
    for (int w = 1; w < 8; ++w) s += sc[w];
    return s;
}

// After the split-KV loop, every thread of every CTA. n partials of request 0 at
// slots slot(e) = (paired ? 2e : e) (the plan CTAs' numbering, as K3 reads them).
// scratch: at least (kMaxParts + 16 * 64 + 64 + 128 + 16) floats of shared memory
// that the loop no longer uses.
__device__ inline void merge_phase(const MlaDecodeParams& p, char* wsb, const WsLayout& ws, int n, bool paired,
                                   float* scratch) {
    FusedSync* sy = reinterpret_cast<FusedSync*>(wsb + ws.sync);
    const ErrSink err = err_sink(p);
    const int t = threadIdx.x;
    const int item = blockIdx.x;
    const bool merges = item < kMergeCtas;
    UvPre uv;
    if (merges) uv_pre(p, item, uv);
    signal(&sy->done);  // this CTA's partials are written

    float* wts = scratch;                  // [kMaxParts] weight of each partial
    float* red = wts + kMaxParts;          // [16][64] sums over partials e = k mod 16
    float* oc = red + 16 * 64;             // [64] o_c over this slice
    float* ys = oc + 64;                   // [128] y of the head (last slice)
    float* sc = ys + 128;                  // [8] warp results, then flags
    int* flag = reinterpret_cast<int*>(sc + 8);
    if (merges) {
        if (t == 0) flag[0] = wait_count(sy, &sy->done, gridDim.x, err) ? 1 : 0;
        __syncthreads();
        MLA_TL_MARK(2, 4);  // every partial written
        if (flag[0]) {
            const int h = item / kFyParts, j = item % kFyParts;
            const float* part_ml = reinterpret_cast<const float*>(wsb + ws.part_ml);
            const float* part_acc = reinterpret_cast<const float*>(wsb + ws.part_acc);
            auto slot = [&](int e) -> int64_t { return paired ? 2 * e : e; };
            // The first burst of partial slices and every (m, L) are requested together (one
            // round trip); M = max over partials with L > 0, w_e = 2^(m_e - M), L = sum w_e L_e.
            // acc over the slice: thread (sub = t >> 4, c4 = t & 15) sums columns [4 c4, 4 c4 + 4)
            // of partials e = sub, sub + 16, ... in order, up to kBurst loads in flight at once;
            // then the 16 subsets are added in subset order.
            constexpr int kBurst = 10;
            const int c4 = t & 15, sub = t >> 4;
            const float4* base = reinterpret_cast<const float4*>(part_acc + (int64_t)h * kLora + 64 * j) + c4;
            const int64_t stride4 = (int64_t)kHeads * kLora / 4;  // float4s between slots
            float4 a[kBurst];
#pragma unroll
            for (int i = 0; i < kBurst; ++i)
                if (sub + 16 * i < n) a[i] = __ldcg(base + slot(sub + 16 * i) * stride4);
            float2 mlr[2];  // e = t, t + 256: every partial (n <= kMaxParts = 512, as the host launches)
#pragma unroll
            for (int k = 0; k < 2; ++k) {
                const int e = t + 256 * k;
                mlr[k] = e < n ? __ldcg(reinterpret_cast<const float2*>(part_ml + (slot(e) * kHeads + h) * 2))
                               : make_float2(-INFINITY, 0.f);
            }
            float mx = -INFINITY;
#pragma unroll
            for (int k = 0; k < 2; ++k)
                if (mlr[k].y > 0.f) mx = fmaxf(mx, mlr[k].x);
            const float M = block_max(mx, sc);
            float ls = 0.f;
#pragma unroll
            for (int k = 0; k < 2; ++k) {
                const int e = t + 256 * k;
                if (e < n) {
                    const float w = mlr[k].y > 0.f ? exp2f(mlr[k].x - M) : 0.f;
                    wts[e] = w;
                    ls = fmaf(w, mlr[k].y, ls);
                }
            }
            const float L = block_sum(ls, sc);  // its barriers also publish wts
            {
                float4 s4 = make_float4(0.f, 0.f, 0.f, 0.f);
                for (int e0 = sub; e0 < n; e0 += 16 * kBurst) {
                    if (e0 != sub) {  // later bursts (more than 160 partials)
#pragma unroll
                        for (int i = 0; i < kBurst; ++i)
                            if (e0 + 16 * i < n) a[i] = __ldcg(base + slot(e0 + 16 * i) * stride4);
                    }
#pragma unroll
                    for (int i = 0; i < kBurst; ++i) {
                        if (e0 + 16 * i < n) {
                            const float wv = wts[e0 + 16 * i];
                            s4.x = fmaf(wv, a[i].x, s4.x);
                            s4.y = fmaf(wv, a[i].y, s4.y);
                            s4.z = fmaf(wv, a[i].z, s4.z);
                            s4.w = fmaf(wv, a[i].w, s4.w);
                        }
                    }
                }
                reinterpret_cast<float4*>(red)[sub * 16 + c4] = s4;
            }
            __syncthreads();
            if (t < 64) {
                const float inv = L > 0.f ? 1.f / L : 0.f;
                float acc = 0.f;
#pragma unroll
                for (int k = 0; k < 16; ++k) acc += red[k * 64 + t];
                oc[t] = acc * inv;
            }
            __syncthreads();
            // y partial: row v = t >> 1 of W_UV[h] over 32 of the slice's columns, pairs summed
            {
                const float* o = oc + 32 * (t & 1);
                float y = 0.f;
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    const __nv_bfloat162* w2 = reinterpret_cast<const __nv_bfloat162*>(&uv.w[k]);
#pragma unroll
                    for (int q = 0; q < 4; ++q) {
                        y = fmaf(o[8 * k + 2 * q], __low2float(w2[q]), y);
                        y = fmaf(o[8 * k + 2 * q + 1], __high2float(w2[q]), y);
                    }
                }
                y += __shfl_xor_sync(0xffffffffu, y, 1);
                float* fy = reinterpret_cast<float*>(wsb + ws.fy);
                if ((t & 1) == 0) fy[(h * kFyParts + j) * kV + (t >> 1)] = y;
            }
            // the last of the head's 8 slices writes the head's result
            __threadfence();
            __syncthreads();
            if (t == 0) flag[1] = atomicAdd(&sy->head[h], 1u) == (uint32_t)(kFyParts - 1) ? 1 : 0;
            __syncthreads();
            if (flag[1]) {
                __threadfence();
                const float* fy = reinterpret_cast<const float*>(wsb + ws.fy);
                if (t < kV) {
                    float y = 0.f;
#pragma unroll
                    for (int jj = 0; jj < kFyParts; ++jj) y += __ldcg(fy + (h * kFyParts + jj) * kV + t);
                    ys[t] = y;
                }
                __syncthreads();
                if (p.world > 0) {  // this shard's (y, m, L) into slot `rank` of every rank's exchange buffer
                    const ExLayout ex = ex_layout(p.world, p.exchange_batch);
                    const uint32_t step = __ldcg(reinterpret_cast<const uint32_t*>(ex_buf(p, p.rank) + ex.ctl)) + 1;
                    if (t <= kV / 2) {
                        for (int d = 0; d < p.world; ++d) {
                            ulonglong2* l = ex_lines(ex_buf(p, d), ex, p.world, p.exchange_batch, step & 1u, p.rank,
                                                     0, h);
                            if (t < kV / 2) st_line(l + t, ys[2 * t], ys[2 * t + 1], step);
                            else st_line(l + kV / 2, M, L, step);
                        }
                    }
                } else if (p.shard_out) {
                    float* so = p.shard_out + (int64_t)h * MLA_SHARD_STRIDE;
                    if (t < kV) so[t] = ys[t];
                    if (t == 0) { so[kV] = M; so[kV + 1] = L; }
                } else if (t < kV) {
                    reinterpret_cast<__nv_bfloat16*>(p.out)[h * kV + t] = __float2bfloat16_rn(ys[t]);
                }
                MLA_TL_MARK(2, 5);  // the head's result written
            }
        }
    }
    // the last CTA out zeroes the counters for the next step
    MLA_TL_EXIT(2);
    __syncthreads();
    if (t == 0 && atomicAdd(&sy->exitc, 1u) == gridDim.x - 1) {
        sy->ready = 0u;
        sy->done = 0u;
        sy->abort = 0u;
#pragma unroll
        for (int h = 0; h < kHeads; ++h) sy->head[h] = 0u;
        __threadfence();
        sy->exitc = 0u;
    }
}

}  // namespace fused
}  // namespace mla
