// K0 — the q | kv_a projection of a decode batch, the step before the
// attention task: q = R(x_n W_q^T), kv_a = R(x_n W_kv_a^T) with the two
// weights stacked as one [3648, 2048] bf16 matrix (reference_decode.py:225-231;
// the reference's fused device task is TASK_QKV_FUSED, fleet_kernel.hip:706-741).
//
// At decode batches the 14.9 MB weight is the whole cost, so the kernel is a
// weight stream: 114 CTAs own 32 weight rows each and request their entire
// 128 KB slice at once (four 32 KB TMA boxes, one per K-quarter), before they
// wait for the previous kernel on the stream (the weight is written by no
// kernel). x_n is staged per block of 16 batch rows by one TMA box that fills
// rows >= B with zeros. Warp w multiplies K-quarter w with m16n8k16 MMAs
// (batch rows on M, weight rows on N, fp32 accumulate); the four quarter sums
// are added in a fixed order and rounded to bf16 once, as a GEMM with fp32
// accumulation rounds its output.
#include <cuda.h>

#include "mla_common.cuh"
#include "mla_mma.cuh"

namespace mla {

namespace k0 {
constexpr int kRows = 32;                        // weight rows per CTA
constexpr int kThreads = 128;                    // 4 warps = 4 K-quarters
constexpr int kQuarter = kHidden / 4;            // 512 columns
constexpr int kWQBytes = kRows * kQuarter * 2;   // 32 KB: [8 column blocks][32 rows][128 B], swizzled
constexpr int kXBytes = 16 * kHidden * 2;        // 64 KB: [32 column blocks][16 rows][128 B], swizzled
constexpr int kRedPitch = 40;                   // floats per batch row of a partial-sum block (no bank conflicts)
constexpr int kRedBytes = 4 * 16 * kRedPitch * 4;  // 10 KB: per-warp partial sums
constexpr int kSmemBytes = 4 * kWQBytes + kXBytes + kRedBytes + 64 + 1024;
static_assert(kQkvRows % kRows == 0, "weight rows must tile by 32");
}  // namespace k0

__global__ void __launch_bounds__(k0::kThreads, 1)
    k0_project(const MlaDecodeParams p, __nv_bfloat16* __restrict__ qkv, const __grid_constant__ CUtensorMap tmap_w,
               const __grid_constant__ CUtensorMap tmap_x) {
    using namespace k0;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* w_s = smem;                          // 4 quarters
    uint8_t* x_s = smem + 4 * kWQBytes;
    float* red = reinterpret_cast<float*>(x_s + kXBytes);
    uint64_t* bar = reinterpret_cast<uint64_t*>(reinterpret_cast<uint8_t*>(red) + kRedBytes);  // [0..3] W, [4] x
    const int n0 = blockIdx.x * kRows;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        for (int i = 0; i < 5; ++i) mbar_init(&bar[i], 1);
        fence_mbar_init();
        prefetch_tmap(&tmap_w);
        prefetch_tmap(&tmap_x);
        for (int qd = 0; qd < 4; ++qd) {  // the weight slice: no kernel writes it, so before pdl_wait
            mbar_arrive_expect_tx(&bar[qd], kWQBytes);
            tma_load_3d(w_s + qd * kWQBytes, &tmap_w, &bar[qd], 0, n0, 8 * qd, kCacheEvictFirst);
        }
    }
    pdl_wait();  // x_n comes from earlier work on the stream
    pdl_trigger();
    __syncthreads();  // barriers initialised

    const int g = lane >> 2, t4 = lane & 3, m8 = lane >> 3, r8 = lane & 7;
    const uint32_t xb = smem_u32(x_s), wb = smem_u32(w_s + warp * kWQBytes);
    const int n_mt = (p.batch + 15) >> 4;
    int dummy = 0;
    for (int mt = 0; mt < n_mt; ++mt) {
        if (threadIdx.x == 0) {  // x_n rows [16 mt, 16 mt + 16), zeros past the batch
            mbar_arrive_expect_tx(&bar[4], kXBytes);
            tma_load_3d(x_s, &tmap_x, &bar[4], 0, 16 * mt, 0, kCacheEvictLast);
        }
        bool ok = mbar_wait(&bar[4], mt & 1, &dummy, p.error_word);
        if (mt == 0) ok = ok && mbar_wait(&bar[warp], 0, &dummy, p.error_word);
        if (!__syncthreads_and(ok)) return;  // a timed-out wait (recorded) ends the whole CTA at once

        float acc[4][4];
#pragma unroll
        for (int n = 0; n < 4; ++n) acc[n][0] = acc[n][1] = acc[n][2] = acc[n][3] = 0.f;
#pragma unroll 4
        for (int ks = 0; ks < kQuarter / 16; ++ks) {
            const int k = kQuarter * warp + 16 * ks;  // column in x_n
            uint32_t a[4];
            {
                const int row = (m8 & 1) * 8 + r8;
                const int unit = ((k & 63) >> 3) + (m8 >> 1);
                ldsm_x4(xb + (k >> 6) * 2048 + row * 128 + ((unit ^ (row & 7)) << 4), a[0], a[1], a[2], a[3]);
            }
            const int kl = 16 * ks;  // column within this warp's quarter
#pragma unroll
            for (int np = 0; np < 2; ++np) {  // weight rows 16 np .. 16 np + 15
                const int n = 16 * np + (m8 >> 1) * 8 + r8;
                const int unit = ((kl & 63) >> 3) + (m8 & 1);
                uint32_t b0, b1, b2, b3;
                ldsm_x4(wb + (kl >> 6) * (kRows * 128) + n * 128 + ((unit ^ (n & 7)) << 4), b0, b1, b2, b3);
                mma16816(acc[2 * np], a, b0, b1);
                mma16816(acc[2 * np + 1], a, b2, b3);
            }
        }
        // quarter sums -> shared memory, [warp][16 batch rows][32 weight rows]
        float* mine = red + warp * 16 * kRedPitch;
#pragma unroll
        for (int n = 0; n < 4; ++n) {
            *reinterpret_cast<float2*>(mine + g * kRedPitch + 8 * n + 2 * t4) = make_float2(acc[n][0], acc[n][1]);
            *reinterpret_cast<float2*>(mine + (g + 8) * kRedPitch + 8 * n + 2 * t4) =
                make_float2(acc[n][2], acc[n][3]);
        }
        __syncthreads();  // every warp has finished with x_s and written its sums
        // 512 outputs of this block: thread -> (batch row, 4 weight rows), quarters added in order
        {
            const int r = threadIdx.x >> 3, c = (threadIdx.x & 7) * 4;
            const int b = 16 * mt + r;
            float v[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const float* e = red + r * kRedPitch + c + j;
                constexpr int q = 16 * kRedPitch;  // one warp's block
                v[j] = ((e[0] + e[q]) + e[2 * q]) + e[3 * q];
            }
            if (b < p.batch) {
                uint2 o;
                o.x = pack_bf16(v[0], v[1]);
                o.y = pack_bf16(v[2], v[3]);
                *reinterpret_cast<uint2*>(qkv + (int64_t)b * kQkvRows + n0 + c) = o;
            }
        }
        __syncthreads();  // red and x_s are reused by the next block of rows
    }
}

cudaError_t k0_configure() {
    return cudaFuncSetAttribute(k0_project, cudaFuncAttributeMaxDynamicSharedMemorySize, k0::kSmemBytes);
}

cudaError_t launch_project(const MlaDecodeParams& p, __nv_bfloat16* qkv, const CUtensorMap& tmap_w,
                           const CUtensorMap& tmap_x, cudaStream_t stream) {
    return launch_pdl(k0_project, dim3(kQkvRows / k0::kRows), dim3(k0::kThreads), k0::kSmemBytes, stream, p, qkv,
                      tmap_w, tmap_x);
}

}  // namespace mla
