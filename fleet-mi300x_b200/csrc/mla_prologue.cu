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
// One 1-D grid with three kinds of CTA:
//   [0, n_absorb)            absorb: (request block of 16, head, 128-column block)
//   [n_absorb, +n_rowwarps)  per-request work, one warp per request
//   last                     planner
#include "mla_common.cuh"

namespace mla {

constexpr int kReqBlock = 16;   // requests per absorb CTA: W_UK tile reuse across requests
constexpr int kColBlock = 128;  // latent columns per absorb CTA
constexpr int kK1Threads = 128;
constexpr int kReqPerRowCta = kK1Threads / 32;

struct K1Grid {
    int n_rb, n_absorb, n_row, total;
    __host__ __device__ explicit K1Grid(int batch) {
        n_rb = (batch + kReqBlock - 1) / kReqBlock;
        n_absorb = n_rb * kHeads * (kLora / kColBlock);
        n_row = (batch + kReqPerRowCta - 1) / kReqPerRowCta;
        total = n_absorb + n_row + 1;
    }
};

// DeepseekV2 RoPE on 64 values x[0..64): interleave-transpose, then rotate_half
// (reference_decode.py:120-134). For pair j < 32:
//   out[j]    = x[2j]*cos[j]       - x[2j+1]*sin[j]
//   out[32+j] = x[2j+1]*cos[32+j]  + x[2j]*sin[32+j]
// Products and the sum are rounded separately, as NumPy evaluates
// `x * cos + rotate_half(x) * sin`.
__device__ __forceinline__ void rope_pair(float x_even, float x_odd, const float* cs, const float* sn, int j,
                                          float& lo, float& hi) {
    lo = __fadd_rn(__fmul_rn(x_even, cs[j]), -__fmul_rn(x_odd, sn[j]));
    hi = __fadd_rn(__fmul_rn(x_odd, cs[32 + j]), __fmul_rn(x_even, sn[32 + j]));
}

__device__ __forceinline__ bool position_ok(const MlaDecodeParams& p, int pos) {
    return pos >= 0 && pos < p.max_pos && pos < p.max_blocks * kPage;
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
            if (!position_ok(p, pos)) record_error(p.error_word, MLA_DEV_BAD_POSITION);
            else n = (pos + 1 + kPage - 1) / kPage;
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

// One warp: kv_post + cache append + q_pe RoPE of request b.
__device__ void request_rows(const MlaDecodeParams& p, __nv_bfloat16* qa, int b, int lane) {
    const int pos = p.seq_lens[b];
    if (!position_ok(p, pos)) return;  // recorded by the planner
    const float* cs = p.rope_cos + (int64_t)pos * kRope;
    const float* sn = p.rope_sin + (int64_t)pos * kRope;
    const __nv_bfloat16* q = reinterpret_cast<const __nv_bfloat16*>(p.q) + (int64_t)b * p.q_stride;
    const __nv_bfloat16* src = reinterpret_cast<const __nv_bfloat16*>(p.kv_a) + (int64_t)b * p.kv_a_stride;
    const __nv_bfloat16* gam = reinterpret_cast<const __nv_bfloat16*>(p.kv_a_norm_w);

    // q_pe of all 16 heads: lane j rotates pair j
    __nv_bfloat16* qrow = qa + (int64_t)b * kQRows * kRow;
#pragma unroll 4
    for (int h = 0; h < kHeads; ++h) {
        const __nv_bfloat162 x = reinterpret_cast<const __nv_bfloat162*>(q + h * kQHead + kNope)[lane];
        float lo, hi;
        rope_pair(__low2float(x), __high2float(x), cs, sn, lane, lo, hi);
        qrow[h * kRow + kLora + lane] = __float2bfloat16_rn(lo);
        qrow[h * kRow + kLora + 32 + lane] = __float2bfloat16_rn(hi);
    }

    // kv_post (reference_decode.py:60-65): var = mean(x^2); y = x * (1 / sqrt(var + eps));
    // row = bf16(bf16(y) * weight). Lane owns c[16*lane, 16*lane+16).
    float x[16];
    {
        const uint4* s4 = reinterpret_cast<const uint4*>(src) + 2 * lane;
        uint4 v[2];
        if ((reinterpret_cast<uintptr_t>(src) & 15) == 0) {
            v[0] = s4[0]; v[1] = s4[1];
            const __nv_bfloat162* h2 = reinterpret_cast<const __nv_bfloat162*>(v);
#pragma unroll
            for (int k = 0; k < 8; ++k) { x[2 * k] = __low2float(h2[k]); x[2 * k + 1] = __high2float(h2[k]); }
        } else {
#pragma unroll
            for (int k = 0; k < 16; ++k) x[k] = __bfloat162float(src[16 * lane + k]);
        }
    }
    float ss = 0.f;
#pragma unroll
    for (int k = 0; k < 16; ++k) ss = __fadd_rn(ss, __fmul_rn(x[k], x[k]));
#pragma unroll
    for (int o = 16; o; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    const float var = __fdiv_rn(ss, (float)kLora);
    const float inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(var, p.rms_eps)));
    __align__(16) __nv_bfloat16 outc[16];
#pragma unroll
    for (int k = 0; k < 16; ++k) {
        const float y = bf16_round(__fmul_rn(x[k], inv));
        outc[k] = __float2bfloat16_rn(__fmul_rn(y, __bfloat162float(gam[16 * lane + k])));
    }
    float lo, hi;
    rope_pair(__bfloat162float(src[kLora + 2 * lane]), __bfloat162float(src[kLora + 2 * lane + 1]), cs, sn, lane,
              lo, hi);
    const int page = p.block_table[(int64_t)b * p.max_blocks + pos / kPage];
    if (page < 0 || page >= p.n_pages) {
        if (lane == 0) record_error(p.error_word, MLA_DEV_BAD_PAGE);
        return;
    }
    __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(p.kv_cache) + ((int64_t)page * kPage + pos % kPage) * kRow;
    reinterpret_cast<uint4*>(dst)[2 * lane] = reinterpret_cast<const uint4*>(outc)[0];
    reinterpret_cast<uint4*>(dst)[2 * lane + 1] = reinterpret_cast<const uint4*>(outc)[1];
    dst[kLora + lane] = __float2bfloat16_rn(lo);
    dst[kLora + 32 + lane] = __float2bfloat16_rn(hi);
}

__global__ void __launch_bounds__(kK1Threads) k1_prologue(const MlaDecodeParams p) {
    const WsLayout ws = ws_layout(p.batch, p.num_ctas);
    char* wsb = reinterpret_cast<char*>(p.workspace);
    __nv_bfloat16* qa = reinterpret_cast<__nv_bfloat16*>(wsb + ws.qa);
    const K1Grid g(p.batch);
    const int cta = blockIdx.x;

    if (cta == g.total - 1) {
        plan_scan(p, reinterpret_cast<int32_t*>(wsb + ws.tiles_cum));
        return;
    }
    if (cta >= g.n_absorb) {
        const int b = (cta - g.n_absorb) * kReqPerRowCta + (threadIdx.x >> 5);
        if (b < p.batch) request_rows(p, qa, b, threadIdx.x & 31);
        return;
    }

    // ---- absorb CTA: q_c[b][h][cols] = q_nope[b][h] @ W_UK[h][:, cols] for 16 requests ----
    __shared__ __align__(16) __nv_bfloat16 w_s[kNope][kColBlock];  // 32 KB
    __shared__ __align__(16) float q_s[kNope][kReqBlock];          // 8 KB, transposed
    const int cb = cta % (kLora / kColBlock);
    const int h = (cta / (kLora / kColBlock)) % kHeads;
    const int rb = cta / (kLora / kColBlock) / kHeads;
    const int b0 = rb * kReqBlock;
    const int nreq = min(kReqBlock, p.batch - b0);
    const __nv_bfloat16* q = reinterpret_cast<const __nv_bfloat16*>(p.q);
    const __nv_bfloat16* kvb = reinterpret_cast<const __nv_bfloat16*>(p.kv_b);
    {
        const uint4* src = reinterpret_cast<const uint4*>(kvb);
        uint4* dst = reinterpret_cast<uint4*>(&w_s[0][0]);
        constexpr int kVecPerRow = kColBlock / 8;
#pragma unroll 4
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
    for (int r = 0; r < kReqBlock; ++r)
        if (r < nreq) qa[((int64_t)(b0 + r) * kQRows + h) * kRow + cb * kColBlock + col] = __float2bfloat16_rn(acc[r]);
}

cudaError_t launch_prologue(const MlaDecodeParams& p, cudaStream_t stream) {
    const K1Grid g(p.batch);
    k1_prologue<<<g.total, kK1Threads, 0, stream>>>(p);
    return cudaGetLastError();
}

}  // namespace mla
