// K3 — merge of the split-KV partials and the W_UV up-projection.
//
// Follows merge_and_uv (src/kernels/attention.h:358-411): global max over the
// partials, rescaled sum in a fixed order, divide by the rescaled sum of
// exps, then o[h] = o_c[h] @ W_UV[h]^T with the bf16 epilogue
// (reference_decode.py:252-256). Partials are merged in CTA order, so the
// result is bitwise reproducible for a fixed split plan.
//
// Grid: x = head, y = block of kMergeReq requests. W_UV[h] (128 x 512 bf16)
// is read once per CTA and reused across the block's requests.
#include "mla_common.cuh"

namespace mla {

constexpr int kMergeReq = 8;
constexpr int kK3Threads = 256;

__global__ void __launch_bounds__(kK3Threads) k3_merge_uv(const MlaDecodeParams p) {
    __shared__ __align__(16) float oc[kMergeReq][kLora];  // 16 KB

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

    // ---- merge: o_c[r][l] = sum_c w_c acc_c[l] / sum_c w_c l_c ----
    for (int r = 0; r < nreq; ++r) {
        const int b = b0 + r;
        const int64_t t0 = cum[b], t1 = cum[b + 1];
        if (t0 == t1) {  // request with an invalid position: zero output
            for (int l = threadIdx.x; l < kLora; l += kK3Threads) oc[r][l] = 0.f;
            continue;
        }
        const int c0 = plan_cta_of(t0, U, G), c1 = plan_cta_of(t1 - 1, U, G);
        float gm = -INFINITY;
        for (int cc = c0; cc <= c1; ++cc) gm = fmaxf(gm, part_ml[((int64_t)(cc + b) * kHeads + h) * 2]);
        float L = 0.f;
        for (int cc = c0; cc <= c1; ++cc) {
            const float* ml = part_ml + ((int64_t)(cc + b) * kHeads + h) * 2;
            L += exp2f(ml[0] - gm) * ml[1];
        }
        const float inv_L = 1.f / L;
        for (int l = threadIdx.x; l < kLora; l += kK3Threads) {
            float v = 0.f;
            for (int cc = c0; cc <= c1; ++cc) {
                const int64_t s = (int64_t)(cc + b) * kHeads + h;
                v = fmaf(exp2f(part_ml[s * 2] - gm), part_acc[s * kLora + l], v);
            }
            oc[r][l] = v * inv_L;
        }
    }
    __syncthreads();

    // ---- out[b][128h + v] = sum_l W_UV[h][v][l] * o_c[r][l] ----
    // warp w takes rows v = w, w+8, ...; lane takes columns [16*lane, 16*lane+16).
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const __nv_bfloat16* wuv = kvb + (int64_t)(h * kKvbHead + kNope) * kLora;
    for (int v = warp; v < kV; v += kK3Threads / 32) {
        const uint4* wrow = reinterpret_cast<const uint4*>(wuv + (int64_t)v * kLora + 16 * lane);
        const uint4 w0 = wrow[0], w1 = wrow[1];
        float wf[16];
        {
            const __nv_bfloat162* a = reinterpret_cast<const __nv_bfloat162*>(&w0);
            const __nv_bfloat162* bb = reinterpret_cast<const __nv_bfloat162*>(&w1);
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const float2 x = __bfloat1622float2(a[k]);
                const float2 y = __bfloat1622float2(bb[k]);
                wf[2 * k] = x.x; wf[2 * k + 1] = x.y;
                wf[8 + 2 * k] = y.x; wf[8 + 2 * k + 1] = y.y;
            }
        }
        float part[kMergeReq];
#pragma unroll
        for (int r = 0; r < kMergeReq; ++r) {
            const float4* o4 = reinterpret_cast<const float4*>(&oc[r][16 * lane]);
            float acc = 0.f;
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                const float4 x = o4[q];
                acc = fmaf(wf[4 * q + 0], x.x, acc);
                acc = fmaf(wf[4 * q + 1], x.y, acc);
                acc = fmaf(wf[4 * q + 2], x.z, acc);
                acc = fmaf(wf[4 * q + 3], x.w, acc);
            }
            part[r] = acc;
        }
#pragma unroll
        for (int r = 0; r < kMergeReq; ++r) {
#pragma unroll
            for (int o = 16; o; o >>= 1) part[r] += __shfl_xor_sync(0xffffffffu, part[r], o);
        }
        if (lane < nreq) {
            float val = 0.f;
#pragma unroll
            for (int r = 0; r < kMergeReq; ++r) if (r == lane) val = part[r];
            out[(int64_t)(b0 + lane) * p.out_stride + h * kV + v] = __float2bfloat16_rn(val);
        }
    }
}

cudaError_t launch_merge_uv(const MlaDecodeParams& p, cudaStream_t stream) {
    dim3 grid(kHeads, (p.batch + kMergeReq - 1) / kMergeReq);
    k3_merge_uv<<<grid, kK3Threads, 0, stream>>>(p);
    return cudaGetLastError();
}

}  // namespace mla
