// K3 — merge of the split-KV partials and the W_UV up-projection.
//
// Follows merge_and_uv (src/kernels/attention.h:358-411): global max over the
// partials, rescaled sum in a fixed order, divide by the rescaled sum of
// exps, then o[h] = o_c[h] @ W_UV[h]^T with the bf16 epilogue
// (reference_decode.py:252-256). Partials are merged in CTA order, so the
// result is bitwise reproducible for a fixed split plan. All in fp32.
//
// Grid: x = head, y = block of kMergeReq requests. Per CTA: the merged o_c of
// the block's requests (transposed, [512][kMergeReq]) and W_UV[h] streamed in
// 64-column chunks through shared memory; each thread owns a 4 (v) x 4
// (request) tile of the [128 x kMergeReq] output.
#include "mla_common.cuh"

namespace mla {

constexpr int kMergeReq = 32;
constexpr int kK3Threads = 256;
constexpr int kOcPitch = kMergeReq + 4;   // floats per latent row of o_c^T (16-byte aligned rows)
constexpr int kWChunk = 64;               // latent columns of W_UV per chunk
constexpr int kWPitch = kWChunk + 2;      // bf16 per W_UV row in shared memory (conflict-free columns)
constexpr int kK3SmemBytes = kLora * kOcPitch * 4 + kV * kWPitch * 2;

__global__ void __launch_bounds__(kK3Threads) k3_merge_uv(const MlaDecodeParams p) {
    extern __shared__ __align__(16) uint8_t smem3[];
    float* ocT = reinterpret_cast<float*>(smem3);                                   // [512][kOcPitch]
    __nv_bfloat16* w_s = reinterpret_cast<__nv_bfloat16*>(ocT + kLora * kOcPitch);  // [128][kWPitch]

    const WsLayout ws = ws_layout(p.batch, p.num_ctas);
    const char* wsb = reinterpret_cast<const char*>(p.workspace);
    const int32_t* cum = reinterpret_cast<const int32_t*>(wsb + ws.tiles_cum);
    const float* part_ml = reinterpret_cast<const float*>(wsb + ws.part_ml);
    const float* part_acc = reinterpret_cast<const float*>(wsb + ws.part_acc);
    const __nv_bfloat16* kvb = reinterpret_cast<const __nv_bfloat16*>(p.kv_b);
    __nv_bfloat16* out = reinterpret_cast<__nv_bfloat16*>(p.out);

    const int h = blockIdx.x;
    const int b0 = blockIdx.y * kMergeReq;
    const int nreq = min(kMergeReq, p.batch - b0);
    const int64_t U = cum[p.batch];
    const int G = (int)(U < 1 ? 1 : (U < (int64_t)p.num_ctas ? U : (int64_t)p.num_ctas));
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    // ---- merge: warp w takes requests w, w+8, ...; lane takes l = lane + 32k ----
    for (int r = warp; r < kMergeReq; r += kK3Threads / 32) {
        float acc[16];
#pragma unroll
        for (int k = 0; k < 16; ++k) acc[k] = 0.f;
        float inv_L = 0.f;
        if (r < nreq) {
            const int b = b0 + r;
            const int64_t t0 = cum[b], t1 = cum[b + 1];
            if (t1 > t0) {  // requests with an invalid position have no tiles: zero output
                const int c0 = plan_cta_of(t0, U, G), c1 = plan_cta_of(t1 - 1, U, G);
                float gm = -INFINITY;
                for (int cc = c0; cc <= c1; ++cc) gm = fmaxf(gm, part_ml[((int64_t)(cc + b) * kHeads + h) * 2]);
                float L = 0.f;
                for (int cc = c0; cc <= c1; ++cc) {
                    const int64_t s = (int64_t)(cc + b) * kHeads + h;
                    const float wgt = exp2f(part_ml[s * 2] - gm);
                    L = fmaf(wgt, part_ml[s * 2 + 1], L);
                    const float* a = part_acc + s * kLora + lane;
#pragma unroll
                    for (int k = 0; k < 16; ++k) acc[k] = fmaf(wgt, a[32 * k], acc[k]);
                }
                inv_L = 1.f / L;
            }
        }
#pragma unroll
        for (int k = 0; k < 16; ++k) ocT[(lane + 32 * k) * kOcPitch + r] = acc[k] * inv_L;
    }

    // ---- out[b][128h + v] = sum_l W_UV[h][v][l] * o_c[r][l] ----
    // thread: v = vl + 32*i (i < 4), r = 4*rg + j (j < 4)
    const int vl = threadIdx.x & 31, rg = threadIdx.x >> 5;
    float o[4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) o[i][j] = 0.f;
    const __nv_bfloat16* wuv = kvb + (int64_t)(h * kKvbHead + kNope) * kLora;
    for (int l0 = 0; l0 < kLora; l0 += kWChunk) {
        __syncthreads();  // previous chunk consumed (and, first time, o_c^T written)
        // W_UV[h][v][l0 : l0+64] -> w_s[v][*]: 128 rows x 8 uint4
        for (int i = threadIdx.x; i < kV * (kWChunk / 8); i += kK3Threads) {
            const int v = i / (kWChunk / 8), c8 = i % (kWChunk / 8);
            const uint4 val = *reinterpret_cast<const uint4*>(wuv + (int64_t)v * kLora + l0 + 8 * c8);
            const uint32_t* u = reinterpret_cast<const uint32_t*>(&val);
            uint32_t* dst = reinterpret_cast<uint32_t*>(w_s + v * kWPitch + 8 * c8);  // 4-byte aligned
#pragma unroll
            for (int k = 0; k < 4; ++k) dst[k] = u[k];
        }
        __syncthreads();
#pragma unroll 8
        for (int l = 0; l < kWChunk; ++l) {
            const float4 oc = *reinterpret_cast<const float4*>(&ocT[(l0 + l) * kOcPitch + 4 * rg]);
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const float w = __bfloat162float(w_s[(vl + 32 * i) * kWPitch + l]);
                o[i][0] = fmaf(w, oc.x, o[i][0]);
                o[i][1] = fmaf(w, oc.y, o[i][1]);
                o[i][2] = fmaf(w, oc.z, o[i][2]);
                o[i][3] = fmaf(w, oc.w, o[i][3]);
            }
        }
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const int r = 4 * rg + j;
        if (r < nreq) {
#pragma unroll
            for (int i = 0; i < 4; ++i)
                out[(int64_t)(b0 + r) * p.out_stride + h * kV + vl + 32 * i] = __float2bfloat16_rn(o[i][j]);
        }
    }
}

cudaError_t k3_configure() {
    return cudaFuncSetAttribute(k3_merge_uv, cudaFuncAttributeMaxDynamicSharedMemorySize, kK3SmemBytes);
}

cudaError_t launch_merge_uv(const MlaDecodeParams& p, cudaStream_t stream) {
    dim3 grid(kHeads, (p.batch + kMergeReq - 1) / kMergeReq);
    k3_merge_uv<<<grid, kK3Threads, kK3SmemBytes, stream>>>(p);
    return cudaGetLastError();
}

}  // namespace mla
