// K0 — the q | kv_a projection of a decode batch, the step before the
// attention task: q = R(x_n W_q^T), kv_a = R(x_n W_kv_a^T) with the two
// weights stacked as one [3648, 2048] bf16 matrix (reference_decode.py:225-231;
// the reference's fused device task is TASK_QKV_FUSED, fleet_kernel.hip:706-741).
// K5 — the step after: h' = R(h + R(W_o R(out))), o_proj with the layer's
// residual add (reference_decode.py:256, 300; TASK_O_PROJ, fleet_kernel.hip:805-824).
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

// Weight-stream GEMM of a decode batch: y[b][n] = epi(sum_k W[n][k] x[b][k]) for
// the N rows of a [N, 2048] bf16 weight, batches of up to 64 rows of x.
//   K0: W = [W_q; W_kv_a] (3648 rows), x = x_n, y = q | kv_a, epi = bf16.
//   K5: W = W_o (2048 rows), x = R(out), y = the new hidden state,
//       epi = bf16(residual + bf16(sum)) (the layer's residual add,
//       reference_decode.py:300; EPI_RESIDUAL of the reference's GEMV, gemv.h:225).
struct StreamArgs {
    __nv_bfloat16* y;
    int64_t y_stride;
    const __nv_bfloat16* residual;  // EPI_RESIDUAL only
    int64_t res_stride;
    int batch;
    ErrSink err;
};

enum StreamEpi { kEpiBf16 = 0, kEpiResidual = 1 };

template <int kRows>
struct WStream {
    static constexpr int kThreads = 128;                    // 4 warps = 4 K-quarters
    static constexpr int kQuarter = kHidden / 4;            // 512 columns
    static constexpr int kWQBytes = kRows * kQuarter * 2;   // [8 column blocks][kRows rows][128 B], swizzled
    static constexpr int kXBytes = 16 * kHidden * 2;        // 64 KB: [32 column blocks][16 rows][128 B], swizzled
    static constexpr int kRedPitch = kRows + 8;             // floats per batch row of a partial-sum block
    static constexpr int kRedBytes = 4 * 16 * kRedPitch * 4;
    static constexpr int kSmemBytes = 4 * kWQBytes + kXBytes + kRedBytes + 64 + 1024;
};

template <int kRows, int kEpi>
__global__ void __launch_bounds__(128, 1)
    k_weight_stream(const StreamArgs a, const __grid_constant__ CUtensorMap tmap_w,
                    const __grid_constant__ CUtensorMap tmap_x) {
    MLA_TL_SCOPE(4);
    using S = WStream<kRows>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* w_s = smem;                          // 4 quarters
    uint8_t* x_s = smem + 4 * S::kWQBytes;
    float* red = reinterpret_cast<float*>(x_s + S::kXBytes);
    uint64_t* bar = reinterpret_cast<uint64_t*>(reinterpret_cast<uint8_t*>(red) + S::kRedBytes);  // [0..3] W, [4] x
    const int n0 = blockIdx.x * kRows;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        for (int i = 0; i < 5; ++i) mbar_init(&bar[i], 1);
        fence_mbar_init();
        prefetch_tmap(&tmap_w);
        prefetch_tmap(&tmap_x);
        for (int qd = 0; qd < 4; ++qd) {  // the weight slice: no kernel writes it, so before pdl_wait
            mbar_arrive_expect_tx(&bar[qd], S::kWQBytes);
            tma_load_3d(w_s + qd * S::kWQBytes, &tmap_w, &bar[qd], 0, n0, 8 * qd, kCacheEvictFirst);
        }
    }
    pdl_wait();  // x (and the residual) come from earlier work on the stream
    MLA_TL_WAITED(4);
    pdl_trigger();
    __syncthreads();  // barriers initialised

    const int g = lane >> 2, t4 = lane & 3, m8 = lane >> 3, r8 = lane & 7;
    const uint32_t xb = smem_u32(x_s), wb = smem_u32(w_s + warp * S::kWQBytes);
    const int n_mt = (a.batch + 15) >> 4;
    int dummy = 0;
    for (int mt = 0; mt < n_mt; ++mt) {
        if (threadIdx.x == 0) {  // x rows [16 mt, 16 mt + 16), zeros past the batch
            mbar_arrive_expect_tx(&bar[4], S::kXBytes);
            tma_load_3d(x_s, &tmap_x, &bar[4], 0, 16 * mt, 0, kCacheEvictLast);
        }
        bool ok = mbar_wait(&bar[4], mt & 1, &dummy, a.err);
        if (mt == 0) ok = ok && mbar_wait(&bar[warp], 0, &dummy, a.err);
        if (!__syncthreads_and(ok)) return;  // a timed-out wait (recorded) ends the whole CTA at once

        constexpr int kNT = kRows / 8;  // n8 tiles of this CTA
        float acc[kNT][4];
#pragma unroll
        for (int n = 0; n < kNT; ++n) acc[n][0] = acc[n][1] = acc[n][2] = acc[n][3] = 0.f;
#pragma unroll 4
        for (int ks = 0; ks < S::kQuarter / 16; ++ks) {
            const int k = S::kQuarter * warp + 16 * ks;  // column of x
            uint32_t af[4];
            {
                const int row = (m8 & 1) * 8 + r8;
                const int unit = ((k & 63) >> 3) + (m8 >> 1);
                ldsm_x4(xb + (k >> 6) * 2048 + row * 128 + ((unit ^ (row & 7)) << 4), af[0], af[1], af[2], af[3]);
            }
            const int kl = 16 * ks;  // column within this warp's quarter
#pragma unroll
            for (int np = 0; np < kNT / 2; ++np) {  // weight rows 16 np .. 16 np + 15
                const int n = 16 * np + (m8 >> 1) * 8 + r8;
                const int unit = ((kl & 63) >> 3) + (m8 & 1);
                uint32_t b0, b1, b2, b3;
                ldsm_x4(wb + (kl >> 6) * (kRows * 128) + n * 128 + ((unit ^ (n & 7)) << 4), b0, b1, b2, b3);
                mma16816(acc[2 * np], af, b0, b1);
                mma16816(acc[2 * np + 1], af, b2, b3);
            }
        }
        // quarter sums -> shared memory, [warp][16 batch rows][kRows weight rows]
        float* mine = red + warp * 16 * S::kRedPitch;
#pragma unroll
        for (int n = 0; n < kNT; ++n) {
            *reinterpret_cast<float2*>(mine + g * S::kRedPitch + 8 * n + 2 * t4) = make_float2(acc[n][0], acc[n][1]);
            *reinterpret_cast<float2*>(mine + (g + 8) * S::kRedPitch + 8 * n + 2 * t4) =
                make_float2(acc[n][2], acc[n][3]);
        }
        __syncthreads();  // every warp has finished with x_s and written its sums
        // 16 x kRows outputs of this block: thread -> (batch row, 4 weight rows), quarters added in order
        for (int o = threadIdx.x; o < 16 * kRows / 4; o += S::kThreads) {
            const int r = o / (kRows / 4), c = (o % (kRows / 4)) * 4;
            const int b = 16 * mt + r;
            if (b >= a.batch) continue;
            float v[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const float* e = red + r * S::kRedPitch + c + j;
                constexpr int q = 16 * S::kRedPitch;  // one warp's block
                v[j] = ((e[0] + e[q]) + e[2 * q]) + e[3 * q];
            }
            if (kEpi == kEpiResidual) {
                const uint2 rv = *reinterpret_cast<const uint2*>(a.residual + (int64_t)b * a.res_stride + n0 + c);
                const __nv_bfloat162* r2 = reinterpret_cast<const __nv_bfloat162*>(&rv);
                v[0] = __low2float(r2[0]) + bf16_round(v[0]);
                v[1] = __high2float(r2[0]) + bf16_round(v[1]);
                v[2] = __low2float(r2[1]) + bf16_round(v[2]);
                v[3] = __high2float(r2[1]) + bf16_round(v[3]);
            }
            uint2 ov;
            ov.x = pack_bf16(v[0], v[1]);
            ov.y = pack_bf16(v[2], v[3]);
            *reinterpret_cast<uint2*>(a.y + (int64_t)b * a.y_stride + n0 + c) = ov;
        }
        __syncthreads();  // red and x_s are reused by the next block of rows
    }
}

constexpr int kK0Rows = 32;   // K0: 3648 / 32 = 114 CTAs
constexpr int kK5Rows = 16;   // K5: 2048 / 16 = 128 CTAs
static_assert(kQkvRows % kK0Rows == 0 && kHidden % kK5Rows == 0, "weight rows must tile");

cudaError_t k0_configure() {
    cudaError_t e = cudaFuncSetAttribute(k_weight_stream<kK0Rows, kEpiBf16>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, WStream<kK0Rows>::kSmemBytes);
    if (e != cudaSuccess) return e;
    return cudaFuncSetAttribute(k_weight_stream<kK5Rows, kEpiResidual>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                WStream<kK5Rows>::kSmemBytes);
}

cudaError_t launch_project(const MlaDecodeParams& p, __nv_bfloat16* qkv, const CUtensorMap& tmap_w,
                           const CUtensorMap& tmap_x, cudaStream_t stream) {
    StreamArgs a{qkv, kQkvRows, nullptr, 0, p.batch, err_sink(p)};
    return launch_pdl(k_weight_stream<kK0Rows, kEpiBf16>, dim3(kQkvRows / kK0Rows), dim3(128),
                      WStream<kK0Rows>::kSmemBytes, stream, a, tmap_w, tmap_x);
}

cudaError_t launch_o_proj(const MlaDecodeParams& p, const CUtensorMap& tmap_w, const CUtensorMap& tmap_x,
                          cudaStream_t stream) {
    StreamArgs a{reinterpret_cast<__nv_bfloat16*>(p.h_out), p.h_out_stride,
                 reinterpret_cast<const __nv_bfloat16*>(p.residual), p.residual_stride, p.batch, err_sink(p)};
    return launch_pdl(k_weight_stream<kK5Rows, kEpiResidual>, dim3(kHidden / kK5Rows), dim3(128),
                      WStream<kK5Rows>::kSmemBytes, stream, a, tmap_w, tmap_x);
}

}  // namespace mla
