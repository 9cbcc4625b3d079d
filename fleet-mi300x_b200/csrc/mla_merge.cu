// K3 — merge of the split-KV partials and the W_UV up-projection.
//
// Follows merge_and_uv (src/kernels/attention.h:358-411): global max over the
// partials, rescaled sum in a fixed order, divide by the rescaled sum of
// exps, then o[h] = o_c[h] @ W_UV[h]^T with the bf16 epilogue
// (reference_decode.py:252-256). Partials are merged in CTA order, so the
// result is bitwise reproducible for a fixed split plan.
//
// Grid: x = head, y = block of 16 requests; 256 threads. The CTA stages
// W_UV[h] (kv_b rows [256h+128, 256h+256), 128 x 512 bf16) with one 128 KB
// TMA box while it merges the partials of its requests into o_c (fp32), then
// runs out[r][v] = sum_l o_c[r][l] W_UV[h][v][l] as m16n8k16 MMAs with the 16
// requests on M. o_c enters the MMA as a bf16 hi/lo pair (hi = bf16(o_c),
// lo = bf16(o_c - hi)), two MMAs per step, so the product keeps ~16 mantissa
// bits of o_c, as the reference's fp32 GEMV does.
#include <cuda.h>

#include "mla_common.cuh"
#include "mla_mma.cuh"

namespace mla {

namespace k3 {
constexpr int kReq = 16;
constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr int kWBytes = kV * kLora * 2;          // 131072: [8 column blocks][128 rows][128 B], swizzled
constexpr int kABytes = kReq * kLora * 2;        // 16384: [16 requests][512] bf16, 1024-byte rows, swizzled
constexpr int kSmemBytes = kWBytes + 2 * kABytes + 64 + 1024;
}  // namespace k3

// Address of element (row, col) of a [rows][512] bf16 matrix stored as 1024-byte
// rows whose 16-byte units are XOR-swizzled with (row & 7) (conflict-free ldmatrix).
__device__ __forceinline__ uint32_t swz1024(uint32_t base, int row, int col) {
    return base + row * 1024 + ((((col >> 3) ^ (row & 7))) << 4) + (col & 7) * 2;
}

__global__ void __launch_bounds__(k3::kThreads, 1)
    k3_merge_uv(const MlaDecodeParams p, const __grid_constant__ CUtensorMap tmap_kvb) {
    using namespace k3;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* w_s = smem;
    uint8_t* a_hi = smem + kWBytes;
    uint8_t* a_lo = a_hi + kABytes;
    uint64_t* bar = reinterpret_cast<uint64_t*>(a_lo + kABytes);

    const WsLayout ws = ws_layout(p.batch, p.num_ctas);
    const char* wsb = reinterpret_cast<const char*>(p.workspace);
    const int32_t* cum = reinterpret_cast<const int32_t*>(wsb + ws.tiles_cum);
    const float* part_ml = reinterpret_cast<const float*>(wsb + ws.part_ml);
    const float* part_acc = reinterpret_cast<const float*>(wsb + ws.part_acc);
    __nv_bfloat16* out = reinterpret_cast<__nv_bfloat16*>(p.out);

    const int h = blockIdx.x;
    const int b0 = blockIdx.y * kReq;
    const int nreq = min(kReq, p.batch - b0);
    const int64_t U = cum[p.batch];
    const int G = (int)(U < 1 ? 1 : (U < (int64_t)p.num_ctas ? U : (int64_t)p.num_ctas));

    if (threadIdx.x == 0) {
        mbar_init(bar, 1);
        fence_mbar_init();
        mbar_arrive_expect_tx(bar, kWBytes);
        tma_load_3d(w_s, &tmap_kvb, bar, 0, h * kKvbHead + kNope, 0, kCacheEvictLast);
    }

    // ---- merge: o_c[r][l] = sum_c w_c acc_c[l] / sum_c w_c l_c ----
    // One pass over the partials in CTA order (running max, rescaled sums); the
    // next partial's loads are issued before the current one is folded in.
    // Warp w merges requests w and w+8; lane owns l = 4 lane + 128 k (k < 4).
    __shared__ int32_t cum_s[kReq + 1];
    if (threadIdx.x <= kReq) cum_s[threadIdx.x] = cum[min(b0 + (int)threadIdx.x, p.batch)];
    __syncthreads();
    const uint32_t ahi = smem_u32(a_hi), alo = smem_u32(a_lo);
    {
        const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
#pragma unroll
        for (int rr = 0; rr < 2; ++rr) {
            const int r = warp + kWarps * rr;
            const int b = b0 + r;
            float4 acc[4];
#pragma unroll
            for (int k = 0; k < 4; ++k) acc[k] = make_float4(0.f, 0.f, 0.f, 0.f);
            float inv_L = 0.f;
            if (r < nreq && cum_s[r + 1] > cum_s[r]) {  // a request with an invalid position has no tiles
                const int c0 = plan_cta_of(cum_s[r], U, G), c1 = plan_cta_of(cum_s[r + 1] - 1, U, G);
                int64_t sidx = (int64_t)(c0 + b) * kHeads + h;
                float2 ml = *reinterpret_cast<const float2*>(part_ml + sidx * 2);
                float4 cur[4];
#pragma unroll
                for (int k = 0; k < 4; ++k) cur[k] = reinterpret_cast<const float4*>(part_acc + sidx * kLora)[lane + 32 * k];
                float m = -INFINITY, L = 0.f;
                for (int cc = c0; cc <= c1; ++cc) {
                    float2 ml_n = ml;
                    float4 nxt[4];
                    if (cc < c1) {
                        const int64_t sn = (int64_t)(cc + 1 + b) * kHeads + h;
                        ml_n = *reinterpret_cast<const float2*>(part_ml + sn * 2);
#pragma unroll
                        for (int k = 0; k < 4; ++k) nxt[k] = reinterpret_cast<const float4*>(part_acc + sn * kLora)[lane + 32 * k];
                    }
                    const float mn = fmaxf(m, ml.x);
                    const float so = exp2f(m - mn), sc = exp2f(ml.x - mn);
                    L = L * so + sc * ml.y;
#pragma unroll
                    for (int k = 0; k < 4; ++k) {
                        acc[k].x = acc[k].x * so + sc * cur[k].x;
                        acc[k].y = acc[k].y * so + sc * cur[k].y;
                        acc[k].z = acc[k].z * so + sc * cur[k].z;
                        acc[k].w = acc[k].w * so + sc * cur[k].w;
                    }
                    m = mn;
                    if (cc < c1) {
                        ml = ml_n;
#pragma unroll
                        for (int k = 0; k < 4; ++k) cur[k] = nxt[k];
                    }
                }
                inv_L = 1.f / L;
            }
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const float o0 = acc[k].x * inv_L, o1 = acc[k].y * inv_L, o2 = acc[k].z * inv_L, o3 = acc[k].w * inv_L;
                const float h0 = bf16_round(o0), h1 = bf16_round(o1), h2 = bf16_round(o2), h3 = bf16_round(o3);
                const int col = 4 * lane + 128 * k;
                uint2 vh, vl;
                vh.x = pack_bf16(h0, h1); vh.y = pack_bf16(h2, h3);
                vl.x = pack_bf16(o0 - h0, o1 - h1); vl.y = pack_bf16(o2 - h2, o3 - h3);
                *reinterpret_cast<uint2*>(a_hi + (swz1024(ahi, r, col) - ahi)) = vh;
                *reinterpret_cast<uint2*>(a_lo + (swz1024(alo, r, col) - alo)) = vl;
            }
        }
    }
    __syncthreads();
    {
        int dummy = 0;
        if (!mbar_wait(bar, 0, &dummy, p.error_word)) return;
    }

    // ---- out[r][v] = sum_l o_c[r][l] W_UV[h][v][l]; warp w owns v in [16w, 16w+16) ----
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g = lane >> 2, t4 = lane & 3, m8 = lane >> 3, r8 = lane & 7;
    const uint32_t wb = smem_u32(w_s);
    float acc[2][4];
#pragma unroll
    for (int n = 0; n < 2; ++n) acc[n][0] = acc[n][1] = acc[n][2] = acc[n][3] = 0.f;
#pragma unroll 4
    for (int ks = 0; ks < kLora / 16; ++ks) {
        uint32_t ah[4], al[4];
        {
            const int row = (m8 & 1) * 8 + r8, col = 16 * ks + (m8 >> 1) * 8;
            ldsm_x4(swz1024(ahi, row, col), ah[0], ah[1], ah[2], ah[3]);
            ldsm_x4(swz1024(alo, row, col), al[0], al[1], al[2], al[3]);
        }
        {  // v tiles 0, 1 of this warp
            const int v = 16 * warp + (m8 >> 1) * 8 + r8;
            const int l = 16 * ks + (m8 & 1) * 8;
            uint32_t b00, b01, b10, b11;
            ldsm_x4(wb + (l >> 6) * (kV * 128) + v * 128 + ((((l & 63) >> 3) ^ r8) << 4), b00, b01, b10, b11);
            mma16816(acc[0], ah, b00, b01);
            mma16816(acc[0], al, b00, b01);
            mma16816(acc[1], ah, b10, b11);
            mma16816(acc[1], al, b10, b11);
        }
    }
#pragma unroll
    for (int n = 0; n < 2; ++n) {
        const int v = 16 * warp + 8 * n + 2 * t4;
        if (g < nreq)
            *reinterpret_cast<uint32_t*>(out + (int64_t)(b0 + g) * p.out_stride + h * kV + v) =
                pack_bf16(acc[n][0], acc[n][1]);
        if (g + 8 < nreq)
            *reinterpret_cast<uint32_t*>(out + (int64_t)(b0 + g + 8) * p.out_stride + h * kV + v) =
                pack_bf16(acc[n][2], acc[n][3]);
    }
}

cudaError_t k3_configure() {
    return cudaFuncSetAttribute(k3_merge_uv, cudaFuncAttributeMaxDynamicSharedMemorySize, k3::kSmemBytes);
}

cudaError_t launch_merge_uv(const MlaDecodeParams& p, const CUtensorMap& tmap_kvb, cudaStream_t stream) {
    dim3 grid(kHeads, (p.batch + k3::kReq - 1) / k3::kReq);
    k3_merge_uv<<<grid, k3::kThreads, k3::kSmemBytes, stream>>>(p, tmap_kvb);
    return cudaGetLastError();
}

}  // namespace mla
