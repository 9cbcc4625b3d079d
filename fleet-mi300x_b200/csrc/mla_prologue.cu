// K1 — the attention task's prologue, once per request (not once per head x
// chunk as in the reference, which re-derives it in every attention task).
//
//  * kv_post: RMSNorm of c_new with HF's two bf16 roundings, RoPE of k_pe_new,
//    bf16 row appended to the request's page (reference_decode.py:231-237,
//    src/kernels/attention.h:62-90);
//  * q_pe RoPE, bf16-rounded (reference_decode.py:235);
//  * q-absorb q_c[h] = q_nope[h] @ W_UK[h] in fp32 (reference_decode.py:250,
//    attention.h:171-216), stored bf16 as the B operand of the tensor-core
//    score contraction;
//  * the split plan: prefix sum of 64-token tiles per request, consumed by K2/K3.
//
// Grid: x = request block of kReqBlock requests (plus one planner CTA),
//       y = head, z = 128-column block of the 512-wide latent.
#include "mla_common.cuh"

namespace mla {

constexpr int kReqBlock = 16;   // requests per absorb CTA: W_UK tile reuse across requests
constexpr int kColBlock = 128;  // latent columns per CTA
constexpr int kK1Threads = 128;

// DeepseekV2 RoPE on 64 values held as x[0..64): interleave-transpose, then
// rotate_half (reference_decode.py:120-134). out[j] for j < 32 and out[32+j]:
//   out[j]    = x[2j]*cos[j]       - x[2j+1]*sin[j]
//   out[32+j] = x[2j+1]*cos[32+j]  + x[2j]*sin[32+j]
// Products and the sum are rounded separately, as NumPy evaluates
// `x * cos + rotate_half(x) * sin`.
__device__ __forceinline__ void rope_pair(float x_even, float x_odd, const float* cs, const float* sn, int j,
                                          float& lo, float& hi) {
    lo = __fadd_rn(__fmul_rn(x_even, cs[j]), -__fmul_rn(x_odd, sn[j]));
    hi = __fadd_rn(__fmul_rn(x_odd, cs[32 + j]), __fmul_rn(x_even, sn[32 + j]));
}

__device__ __forceinline__ float block_sum_128(float v, float* red) {
#pragma unroll
    for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    __syncthreads();
    if (lane == 0) red[warp] = v;
    __syncthreads();
    return (red[0] + red[1]) + (red[2] + red[3]);  // fixed order
}

// Prefix sum of tiles per request (one CTA). Invalid positions are recorded
// and given zero tiles, so no later kernel reads outside the block table.
__device__ void plan_scan(const MlaDecodeParams& p, int32_t* cum) {
    __shared__ int32_t warp_tot[kK1Threads / 32];
    __shared__ int32_t carry;
    if (threadIdx.x == 0) carry = 0;
    __syncthreads();
    for (int base = 0; base < p.batch; base += kK1Threads) {
        const int b = base + threadIdx.x;
        int n = 0;
        if (b < p.batch) {
            const int pos = p.seq_lens[b];
            if (pos < 0 || pos >= p.max_pos || pos >= p.max_blocks * kPage) {
                record_error(p.error_word, MLA_DEV_BAD_POSITION);
            } else {
                n = (pos + 1 + kPage - 1) / kPage;
            }
        }
        int incl = n;
        const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int t = __shfl_up_sync(0xffffffffu, incl, o);
            if (lane >= o) incl += t;
        }
        if (lane == 31) warp_tot[warp] = incl;
        __syncthreads();
        int before = carry;
        for (int w = 0; w < warp; ++w) before += warp_tot[w];
        if (b < p.batch) cum[b] = before + incl - n;
        __syncthreads();
        if (threadIdx.x == kK1Threads - 1) carry = before + incl;
        __syncthreads();
    }
    if (threadIdx.x == 0) cum[p.batch] = carry;
}

__global__ void __launch_bounds__(kK1Threads) k1_prologue(const MlaDecodeParams p) {
    const WsLayout ws = ws_layout(p.batch, p.num_ctas);
    char* wsb = reinterpret_cast<char*>(p.workspace);
    const int n_rb = (p.batch + kReqBlock - 1) / kReqBlock;

    if (blockIdx.x == n_rb) {  // planner CTA
        if (blockIdx.y == 0 && blockIdx.z == 0) plan_scan(p, reinterpret_cast<int32_t*>(wsb + ws.tiles_cum));
        return;
    }

    __shared__ __align__(16) __nv_bfloat16 w_s[kNope][kColBlock];  // W_UK[h][:, cols], 32 KB
    __shared__ __align__(16) float q_s[kNope][kReqBlock];          // q_nope, transposed, 8 KB
    __shared__ float red[4];
    __shared__ float row_s[kRow];

    const int h = blockIdx.y, cb = blockIdx.z;
    const int b0 = blockIdx.x * kReqBlock;
    const int nreq = min(kReqBlock, p.batch - b0);
    const __nv_bfloat16* q = reinterpret_cast<const __nv_bfloat16*>(p.q);
    const __nv_bfloat16* kvb = reinterpret_cast<const __nv_bfloat16*>(p.kv_b);
    __nv_bfloat16* qa = reinterpret_cast<__nv_bfloat16*>(wsb + ws.qa);

    // ---- stage W_UK[h][0:128, cb*128 : cb*128+128] (kv_b rows 256h + d) ----
    {
        const uint4* src = reinterpret_cast<const uint4*>(kvb);
        uint4* dst = reinterpret_cast<uint4*>(&w_s[0][0]);
        constexpr int kVecPerRow = kColBlock / 8;  // 16
        for (int i = threadIdx.x; i < kNope * kVecPerRow; i += kK1Threads) {
            const int d = i / kVecPerRow, v = i % kVecPerRow;
            dst[i] = src[((int64_t)(h * kKvbHead + d) * kLora + cb * kColBlock) / 8 + v];
        }
    }
    for (int i = threadIdx.x; i < kNope * kReqBlock; i += kK1Threads) {
        const int r = i / kNope, d = i % kNope;
        q_s[d][r] = r < nreq ? __bfloat162float(q[(int64_t)(b0 + r) * p.q_stride + h * kQHead + d]) : 0.f;
    }
    __syncthreads();

    // ---- q_c[b][h][col] = sum_d q_nope[b][h][d] * W_UK[h][d][col], fp32 ----
    {
        const int col = threadIdx.x;
        float acc[kReqBlock];
#pragma unroll
        for (int r = 0; r < kReqBlock; ++r) acc[r] = 0.f;
#pragma unroll 4
        for (int d = 0; d < kNope; ++d) {
            const float w = __bfloat162float(w_s[d][col]);
            const float4* q4 = reinterpret_cast<const float4*>(&q_s[d][0]);
#pragma unroll
            for (int r4 = 0; r4 < kReqBlock / 4; ++r4) {
                const float4 qq = q4[r4];
                acc[4 * r4 + 0] = fmaf(qq.x, w, acc[4 * r4 + 0]);
                acc[4 * r4 + 1] = fmaf(qq.y, w, acc[4 * r4 + 1]);
                acc[4 * r4 + 2] = fmaf(qq.z, w, acc[4 * r4 + 2]);
                acc[4 * r4 + 3] = fmaf(qq.w, w, acc[4 * r4 + 3]);
            }
        }
#pragma unroll
        for (int r = 0; r < kReqBlock; ++r) {
            if (r < nreq) {
                qa[((int64_t)(b0 + r) * kQRows + h) * kRow + cb * kColBlock + col] = __float2bfloat16_rn(acc[r]);
            }
        }
    }

    if (cb != 0) return;

    // ---- q_pe RoPE for head h (cb == 0 CTAs) ----
    for (int r = 0; r < nreq; ++r) {
        const int b = b0 + r;
        const int pos = p.seq_lens[b];
        if (pos < 0 || pos >= p.max_pos) continue;  // recorded by the planner
        const float* cs = p.rope_cos + (int64_t)pos * kRope;
        const float* sn = p.rope_sin + (int64_t)pos * kRope;
        if (threadIdx.x < 32) {
            const int j = threadIdx.x;
            const __nv_bfloat16* qp = q + (int64_t)b * p.q_stride + h * kQHead + kNope;
            float lo, hi;
            rope_pair(__bfloat162float(qp[2 * j]), __bfloat162float(qp[2 * j + 1]), cs, sn, j, lo, hi);
            __nv_bfloat16* dst = qa + ((int64_t)b * kQRows + h) * kRow + kLora;
            dst[j] = __float2bfloat16_rn(lo);
            dst[32 + j] = __float2bfloat16_rn(hi);
        }
    }

    if (h != 0) return;

    // ---- kv_post for the block's requests (h == 0, cb == 0) ----
    const __nv_bfloat16* kva = reinterpret_cast<const __nv_bfloat16*>(p.kv_a);
    const __nv_bfloat16* gam = reinterpret_cast<const __nv_bfloat16*>(p.kv_a_norm_w);
    __nv_bfloat16* cache = reinterpret_cast<__nv_bfloat16*>(p.kv_cache);
    for (int r = 0; r < nreq; ++r) {
        const int b = b0 + r;
        const int pos = p.seq_lens[b];
        const bool pos_ok = pos >= 0 && pos < p.max_pos && pos < p.max_blocks * kPage;
        const __nv_bfloat16* src = kva + (int64_t)b * p.kv_a_stride;
        float ss = 0.f;
        for (int i = threadIdx.x; i < kLora; i += kK1Threads) {
            const float v = __bfloat162float(src[i]);
            ss = fmaf(v, v, ss);
        }
        const float sumsq = block_sum_128(ss, red);
        // reference_decode.py:60-65: var = mean(x^2); y = x * (1 / sqrt(var + eps));
        // bf16(y) * weight, rounded to bf16 again.
        const float var = __fdiv_rn(sumsq, (float)kLora);
        const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(var, p.rms_eps)));
        for (int i = threadIdx.x; i < kLora; i += kK1Threads) {
            const float y = bf16_round(__fmul_rn(__bfloat162float(src[i]), inv));
            row_s[i] = bf16_round(__fmul_rn(y, __bfloat162float(gam[i])));
        }
        if (pos_ok && threadIdx.x < 32) {
            const int j = threadIdx.x;
            const float* cs = p.rope_cos + (int64_t)pos * kRope;
            const float* sn = p.rope_sin + (int64_t)pos * kRope;
            float lo, hi;
            rope_pair(__bfloat162float(src[kLora + 2 * j]), __bfloat162float(src[kLora + 2 * j + 1]), cs, sn, j,
                      lo, hi);
            row_s[kLora + j] = lo;
            row_s[kLora + 32 + j] = hi;
        }
        __syncthreads();
        if (pos_ok) {
            const int page = p.block_table[(int64_t)b * p.max_blocks + pos / kPage];
            if (page < 0 || page >= p.n_pages) {
                if (threadIdx.x == 0) record_error(p.error_word, MLA_DEV_BAD_PAGE);
            } else {
                __nv_bfloat16* dst = cache + ((int64_t)page * kPage + pos % kPage) * kRow;
                for (int i = threadIdx.x; i < kRow; i += kK1Threads) dst[i] = __float2bfloat16_rn(row_s[i]);
            }
        }
        __syncthreads();
    }
}

cudaError_t launch_prologue(const MlaDecodeParams& p, cudaStream_t stream) {
    const int n_rb = (p.batch + kReqBlock - 1) / kReqBlock;
    dim3 grid(n_rb + 1, kHeads, kLora / kColBlock);
    k1_prologue<<<grid, kK1Threads, 0, stream>>>(p);
    return cudaGetLastError();
}

}  // namespace mla
