// K2 (default) — split-KV absorbed-MLA attention with exactly 16 heads on the
// MMA's M dimension: mma.sync m16n8k16 (bf16 in, fp32 accumulate) fed by
// whole-page TMA tiles.
//
// Why this shape: with 16 heads and one query per request the contractions
// are [16 x 576] x [576 x tokens] (scores) and [16 x tokens] x [tokens x 512]
// (output). A 5th-generation (tcgen05) MMA costs the same issue slot whatever
// its N, so at N = 16 it runs ~16x below its rate and the score contraction
// alone (36 MMAs per 64-token page) cannot keep up with HBM; m16n8k16 has M =
// 16 = heads exactly and sustains ~2 cycles per instruction per SM, so a page
// (544 MMAs, 2.2 MFLOP) costs ~0.6 us against ~1.6 us of HBM time. The
// tensor-memory kernel (mla_attention.cu) stays available for comparison.
//
// Per CTA (one per SM), 160 threads:
//   warp 0      TMA producer: one 4-D box per 64-token page (72 KB), landing
//               as 9 swizzled [64 tokens x 64 columns] blocks, 2-slot ring.
//   warps 1-4   compute warp w (0..3):
//     scores    S_w = Q[:, 144w : 144w+144] C[:, 144w : 144w+144]^T for all 64
//               tokens (9 k-steps x 8 token tiles), Q fragments in registers;
//     exchange  the 4 partial S through shared memory; warp w sums the 16
//               tokens [16w, 16w+16) and runs the softmax on them;
//     softmax   lazy rescale: the running max per head is kept unless a score
//               exceeds it by more than 2^8 (one barrier-reduction decides),
//               probabilities rounded to bf16 and shared through shared memory;
//     output    O_w[16 x 128] += P[16 x 64] C[:, 128w : 128w+128] (4 k-steps x
//               16 latent tiles), accumulated in registers (rescale = multiply).
// The split plan and the partial layout are the same as the other K2 kernels
// (mla_tiles.cuh), so K3 merges any of them.
#include <cuda.h>

#include "mla_common.cuh"
#include "mla_tiles.cuh"
#include "mla_mma.cuh"

namespace mla {

namespace mmak {

constexpr int kThreads = 160;
constexpr int kWarps = 4;                    // compute warps
constexpr int kNTile = 2;                    // whole-page ring
constexpr int kChunkBytes = 8192;
constexpr int kTileBytes = 9 * kChunkBytes;
constexpr int kSPitch = 72;                  // floats per head row of a partial-score block (64-bit
                                             // accesses by a half-warp then hit 32 distinct banks)
constexpr int kSPartBytes = kWarps * kHeads * kSPitch * 4;   // 17,408
constexpr int kPBytes = kHeads * 128;        // [16 heads][64 tokens] bf16, 128-byte swizzled rows

struct Smem {
    uint64_t tile_full[kNTile], tile_empty[kNTile];
    int abort;
    float tmax[kWarps][16];
    float lsum[kWarps][16];
};

constexpr int kOffTile = 0;
constexpr int kOffS = kOffTile + kNTile * kTileBytes;
constexpr int kOffP = kOffS + kSPartBytes;
constexpr int kOffMisc = kOffP + 2 * kPBytes;
constexpr int kSmemBytes = kOffMisc + (int)sizeof(Smem) + 1024;
static_assert(kSmemBytes <= 232448, "K2 (mma) shared memory exceeds 227 KB");

// Zero the bf16 halves of a B fragment register whose token index is >= valid.
__device__ __forceinline__ uint32_t mask_pair(uint32_t v, int tok_lo, int valid) {
    if (tok_lo >= valid) return 0u;
    if (tok_lo + 1 >= valid) return v & 0x0000FFFFu;
    return v;
}

}  // namespace mmak

__global__ void __launch_bounds__(mmak::kThreads, 1)
    k2_attention_mma(const MlaDecodeParams p, const __grid_constant__ CUtensorMap tmap_kv, float scale_log2) {
    using namespace mmak;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    Smem& S = *reinterpret_cast<Smem*>(smem + kOffMisc);
    uint8_t* tile_s = smem + kOffTile;
    float* spart = reinterpret_cast<float*>(smem + kOffS);
    uint8_t* p_s = smem + kOffP;

    const WsLayout ws = ws_layout(p);
    char* wsb = reinterpret_cast<char*>(p.workspace);
    const int32_t* cum = reinterpret_cast<const int32_t*>(wsb + ws.tiles_cum);
    const __nv_bfloat16* qa = reinterpret_cast<const __nv_bfloat16*>(wsb + ws.qa);
    float* part_ml = reinterpret_cast<float*>(wsb + ws.part_ml);
    float* part_acc = reinterpret_cast<float*>(wsb + ws.part_acc);

    pdl_trigger();
    pdl_wait();  // the plan, absorbed queries and new rows come from K1
    const int64_t U = cum[p.batch];
    const int G = (int)(U < (int64_t)p.num_ctas ? U : (int64_t)p.num_ctas);
    const int c = blockIdx.x;
    if (c >= G) return;
    const int64_t u_begin = plan_begin(c, U, G), u_end = plan_begin(c + 1, U, G);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        for (int i = 0; i < kNTile; ++i) { mbar_init(&S.tile_full[i], 1); mbar_init(&S.tile_empty[i], kWarps); }
        S.abort = 0;
        fence_mbar_init();
    }
    __syncthreads();
    volatile int* abort = &S.abort;

    TileCursor cur;
    cur.init(cum, p.seq_lens, p.batch, u_begin, u_end, new_row_count(p));

    if (warp == 0) {
        // ------------------------------------------------------------ producer
        if (lane == 0) {
            prefetch_tmap(&tmap_kv);
            uint32_t t = 0;
            for (; cur.valid(); cur.next(), ++t) {
                int page = p.block_table[(int64_t)cur.b * p.max_blocks + cur.page_index()];
                if (page < 0 || page >= p.n_pages) { record_error(p.error_word, MLA_DEV_BAD_PAGE); page = 0; }
                const uint32_t slot = t % kNTile, n = t / kNTile;
                if (n > 0 && !mbar_wait_idle(&S.tile_empty[slot], (n - 1) & 1, abort, p.error_word)) break;
                mbar_arrive_expect_tx(&S.tile_full[slot], kTileBytes);
                tma_load_4d(tile_s + slot * kTileBytes, &tmap_kv, &S.tile_full[slot], 0, 0, 0, page, kCacheEvictFirst);
            }
            for (uint32_t sl = 0; sl < kNTile; ++sl) {
                const uint32_t fills = t / kNTile + (sl < t % kNTile ? 1u : 0u);
                if (fills) mbar_drain(&S.tile_full[sl], (fills - 1) & 1, p.error_word);
            }
        }
    } else {
        // ------------------------------------------------------------ compute warps
        const int w = warp - 1;                // 0..3
        const int g = lane >> 2, t4 = lane & 3;
        const int m8 = lane >> 3, r8 = lane & 7;  // ldmatrix: matrix index, row in matrix
        const int cw_tid = threadIdx.x - 32;
        const uint32_t tile_addr = smem_u32(tile_s), p_addr = smem_u32(p_s);

        uint32_t qf[9][4];                     // Q fragments, k-steps [9w, 9w+9)
        float o[16][4];                        // O_w: 16 latent tiles of 8
        float m_run[2], l_run[2];              // heads g, g+8
        int rows_b = 0;                        // rows attended by the current request (seq_lens[b] + 1)
        int i = 0;
        for (; cur.valid(); cur.next(), ++i) {
            const bool first = cur.first(), last = cur.last();
            if (first) rows_b = p.seq_lens[cur.b] + new_row_count(p);
            const int valid = min(kPage, rows_b - cur.page_index() * kPage);
            if (first) {
                const __nv_bfloat16* qrow = qa + (int64_t)cur.b * kQRows * kRow + 144 * w + 2 * t4;
#pragma unroll
                for (int j = 0; j < 9; ++j) {
                    const __nv_bfloat16* q0 = qrow + 16 * j;
                    qf[j][0] = *reinterpret_cast<const uint32_t*>(q0 + g * kRow);
                    qf[j][1] = *reinterpret_cast<const uint32_t*>(q0 + (g + 8) * kRow);
                    qf[j][2] = *reinterpret_cast<const uint32_t*>(q0 + g * kRow + 8);
                    qf[j][3] = *reinterpret_cast<const uint32_t*>(q0 + (g + 8) * kRow + 8);
                }
#pragma unroll
                for (int n = 0; n < 16; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;
                m_run[0] = m_run[1] = -INFINITY;
                l_run[0] = l_run[1] = 0.f;
            }
            const uint32_t slot = (uint32_t)i % kNTile;
            if (!mbar_wait(&S.tile_full[slot], ((uint32_t)i / kNTile) & 1, abort, p.error_word)) break;
            const uint32_t tbase = tile_addr + slot * kTileBytes;

            // ---- partial scores over this warp's 144 columns, all 64 tokens ----
            float sacc[8][4];
#pragma unroll
            for (int n = 0; n < 8; ++n) sacc[n][0] = sacc[n][1] = sacc[n][2] = sacc[n][3] = 0.f;
#pragma unroll
            for (int j = 0; j < 9; ++j) {
                const int k = 144 * w + 16 * j;
                const int chunk = k >> 6, unit = ((k & 63) >> 3) + (m8 & 1);
#pragma unroll
                for (int q = 0; q < 4; ++q) {  // token tiles 2q, 2q+1
                    const int tok = 16 * q + (m8 >> 1) * 8 + r8;
                    uint32_t b00, b01, b10, b11;
                    ldsm_x4(tbase + chunk * kChunkBytes + tok * 128 + ((unit ^ r8) << 4), b00, b01, b10, b11);
                    mma16816(sacc[2 * q], qf[j], b00, b01);
                    mma16816(sacc[2 * q + 1], qf[j], b10, b11);
                }
            }
            // ---- exchange: every warp publishes its partials, then sums its 16 tokens ----
            {
                float* mine = spart + w * (kHeads * kSPitch);
#pragma unroll
                for (int n = 0; n < 8; ++n) {
                    *reinterpret_cast<float2*>(mine + g * kSPitch + 8 * n + 2 * t4) = make_float2(sacc[n][0], sacc[n][1]);
                    *reinterpret_cast<float2*>(mine + (g + 8) * kSPitch + 8 * n + 2 * t4) =
                        make_float2(sacc[n][2], sacc[n][3]);
                }
            }
            named_bar_sync(1, 128);
            float s[2][4];  // token tile n' (tokens 16w + 8n' + 2t4 + {0,1}); [0..1] head g, [2..3] head g+8
#pragma unroll
            for (int n = 0; n < 2; ++n) {
                const int col = 16 * w + 8 * n + 2 * t4;
                float2 lo = make_float2(0.f, 0.f), hi = make_float2(0.f, 0.f);
#pragma unroll
                for (int v = 0; v < kWarps; ++v) {
                    const float* part = spart + v * (kHeads * kSPitch);
                    const float2 a = *reinterpret_cast<const float2*>(part + g * kSPitch + col);
                    const float2 b = *reinterpret_cast<const float2*>(part + (g + 8) * kSPitch + col);
                    lo.x += a.x; lo.y += a.y; hi.x += b.x; hi.y += b.y;
                }
                const int tk = col;  // token index of element 0
                s[n][0] = tk < valid ? lo.x * scale_log2 : -INFINITY;
                s[n][1] = tk + 1 < valid ? lo.y * scale_log2 : -INFINITY;
                s[n][2] = tk < valid ? hi.x * scale_log2 : -INFINITY;
                s[n][3] = tk + 1 < valid ? hi.y * scale_log2 : -INFINITY;
            }
            // ---- running max (log2 domain), lazy rescale ----
            bool exchange = first;
            if (!first) {
                const bool ex = fmaxf(fmaxf(s[0][0], s[0][1]), fmaxf(s[1][0], s[1][1])) > m_run[0] + 8.f ||
                                fmaxf(fmaxf(s[0][2], s[0][3]), fmaxf(s[1][2], s[1][3])) > m_run[1] + 8.f;
                exchange = bar_red_or(1, 128, ex);
            }
            if (exchange) {
                float mx0 = fmaxf(fmaxf(s[0][0], s[0][1]), fmaxf(s[1][0], s[1][1]));
                float mx1 = fmaxf(fmaxf(s[0][2], s[0][3]), fmaxf(s[1][2], s[1][3]));
                mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
                mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
                mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
                mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
                if (t4 == 0) { S.tmax[w][g] = mx0; S.tmax[w][g + 8] = mx1; }
                named_bar_sync(1, 128);
                const float t0 = fmaxf(fmaxf(S.tmax[0][g], S.tmax[1][g]), fmaxf(S.tmax[2][g], S.tmax[3][g]));
                const float t1 = fmaxf(fmaxf(S.tmax[0][g + 8], S.tmax[1][g + 8]), fmaxf(S.tmax[2][g + 8], S.tmax[3][g + 8]));
                const float n0 = fmaxf(m_run[0], t0), n1 = fmaxf(m_run[1], t1);
                if (!first) {
                    const float f0 = fast_exp2(m_run[0] - n0), f1 = fast_exp2(m_run[1] - n1);
#pragma unroll
                    for (int n = 0; n < 16; ++n) { o[n][0] *= f0; o[n][1] *= f0; o[n][2] *= f1; o[n][3] *= f1; }
                    l_run[0] *= f0;
                    l_run[1] *= f1;
                }
                m_run[0] = n0;
                m_run[1] = n1;
            }
            // ---- probabilities (bf16) for this warp's 16 tokens -> P buffer ----
            uint8_t* pb = p_s + (i & 1) * kPBytes;
#pragma unroll
            for (int n = 0; n < 2; ++n) {
                const float e0 = bf16_round(fast_exp2(s[n][0] - m_run[0]));
                const float e1 = bf16_round(fast_exp2(s[n][1] - m_run[0]));
                const float e2 = bf16_round(fast_exp2(s[n][2] - m_run[1]));
                const float e3 = bf16_round(fast_exp2(s[n][3] - m_run[1]));
                l_run[0] += e0 + e1;
                l_run[1] += e2 + e3;
                const int unit = 2 * w + n;  // token / 8
                *reinterpret_cast<uint32_t*>(pb + g * 128 + ((unit ^ (g & 7)) << 4) + 4 * t4) = pack_bf16(e0, e1);
                *reinterpret_cast<uint32_t*>(pb + (g + 8) * 128 + ((unit ^ (g & 7)) << 4) + 4 * t4) = pack_bf16(e2, e3);
            }
            named_bar_sync(1, 128);

            // ---- O_w += P C[:, 128w : 128w+128] ----
            const uint32_t pbase = p_addr + (i & 1) * kPBytes;
#pragma unroll
            for (int ks = 0; ks < 4; ++ks) {
                uint32_t a[4];
                {
                    const int head = (m8 & 1) * 8 + r8;
                    const int unit = 2 * ks + (m8 >> 1);
                    ldsm_x4(pbase + head * 128 + ((unit ^ r8) << 4), a[0], a[1], a[2], a[3]);
                }
                const int tok = 16 * ks + (m8 & 1) * 8 + r8;
#pragma unroll
                for (int pp = 0; pp < 8; ++pp) {  // latent tiles 2pp, 2pp+1 of this warp
                    const int chunk = 2 * w + (pp >> 2);
                    const int unit = 2 * (pp & 3) + (m8 >> 1);
                    uint32_t b00, b01, b10, b11;
                    ldsm_x4_t(tbase + chunk * kChunkBytes + tok * 128 + ((unit ^ r8) << 4), b00, b01, b10, b11);
                    if (valid < kPage) {
                        const int tl = 16 * ks + 2 * t4;
                        b00 = mask_pair(b00, tl, valid);
                        b10 = mask_pair(b10, tl, valid);
                        b01 = mask_pair(b01, tl + 8, valid);
                        b11 = mask_pair(b11, tl + 8, valid);
                    }
                    mma16816(o[2 * pp], a, b00, b01);
                    mma16816(o[2 * pp + 1], a, b10, b11);
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&S.tile_empty[slot]);

            if (last) {
                // ---- partial of (request, this CTA): m, l, unnormalised O ----
                float l0 = l_run[0], l1 = l_run[1];
                l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
                l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
                l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
                l1 += __shfl_xor_sync(0xffffffffu, l1, 2);
                if (t4 == 0) { S.lsum[w][g] = l0; S.lsum[w][g + 8] = l1; }
                named_bar_sync(1, 128);
                const int64_t slot_idx = (int64_t)c + cur.b;
                if (w == 0 && t4 == 0) {
                    const float L0 = (S.lsum[0][g] + S.lsum[1][g]) + (S.lsum[2][g] + S.lsum[3][g]);
                    const float L1 = (S.lsum[0][g + 8] + S.lsum[1][g + 8]) + (S.lsum[2][g + 8] + S.lsum[3][g + 8]);
                    part_ml[(slot_idx * kHeads + g) * 2 + 0] = m_run[0];
                    part_ml[(slot_idx * kHeads + g) * 2 + 1] = L0;
                    part_ml[(slot_idx * kHeads + g + 8) * 2 + 0] = m_run[1];
                    part_ml[(slot_idx * kHeads + g + 8) * 2 + 1] = L1;
                }
                float* acc = part_acc + slot_idx * kHeads * kLora + 128 * w + 2 * t4;
#pragma unroll
                for (int n = 0; n < 16; ++n) {
                    *reinterpret_cast<float2*>(acc + g * kLora + 8 * n) = make_float2(o[n][0], o[n][1]);
                    *reinterpret_cast<float2*>(acc + (g + 8) * kLora + 8 * n) = make_float2(o[n][2], o[n][3]);
                }
                // the lsum buffer is reused by the next segment's epilogue only after
                // at least one more tile's barriers, which every warp passes after this read
            }
        }
        (void)cw_tid;
    }
    __syncthreads();
}

int k2_mma_smem_bytes() { return mmak::kSmemBytes; }

cudaError_t k2_mma_configure() {
    return cudaFuncSetAttribute(k2_attention_mma, cudaFuncAttributeMaxDynamicSharedMemorySize, mmak::kSmemBytes);
}

cudaError_t launch_attention_mma(const MlaDecodeParams& p, const CUtensorMap& tmap_kv, float scale_log2,
                                 cudaStream_t stream) {
    const cudaError_t e = launch_pdl(k2_attention_mma, dim3(p.num_ctas), dim3(mmak::kThreads), mmak::kSmemBytes,
                                     stream, p, tmap_kv, scale_log2);
    if (e != cudaSuccess) return e;
    return cudaGetLastError();
}

}  // namespace mla
