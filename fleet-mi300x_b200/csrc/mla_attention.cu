// K2 — split-KV absorbed-MLA attention over the paged latent cache.
//
// The reference's attention_chunk (src/kernels/attention.h:230-351) runs one
// workgroup per (head, chunk) and so reads every cache row once per head
// (16x). Here one CTA serves all 16 heads of a request, so each 1152-byte
// latent row is brought from HBM into shared memory exactly once, and both
// contractions run on the 5th-generation tensor cores with the token axis on
// the MMA's M dimension and the 16 heads on N:
//
//   scores  S^T[t][h]  = sum_k C[t][k] * Qa[h][k]       (k over 576 = c_kv | k_pe)
//   output  O^T[l][h] += sum_t C[t][l] * P^T[t][h]      (l over the 512 latent columns)
//
// Qa = q_c | q_pe (absorbed query, from K1). S^T lives in TMEM as a 64-lane x
// 16-column fp32 tile per 64-token page (M = 64), O^T as four 128-lane x
// 16-column blocks (M = 128). A page tile is staged by TMA in 128-byte
// swizzled 64x64 boxes; the same shared-memory bytes serve as the K-major A
// operand of the score MMA and the MN-major A operand of the output MMA.
//
// Work split (the split-KV scheduler): the pages of all requests form one
// list, cut into num_ctas equal ranges; CTA c writes one partial
// (m, l, acc[512]) per (request, head) it touches, at slot c + b. K3 merges
// them in CTA order, so results are bitwise reproducible for a fixed
// num_ctas (the reference's fixed-order merge rule, docs/design.md:148).
//
// Warp roles (192 threads):
//   warp 0     TMA producer (one thread)
//   warp 1     TMEM owner + tcgen05.mma issuer (one thread)
//   warps 2-5  softmax / epilogue; warp w owns TMEM lanes 32*(w%4)..+32
// Every wait is bounded (mla::mbar_wait): a stall records MLA_DEV_TIMEOUT
// and the CTA drains its copies, frees TMEM and returns.
#include <cuda.h>

#include "mla_common.cuh"

namespace mla {

constexpr int kK2Threads = 192;
constexpr int kNPair = 10;                   // ring of 16 KB slots: 64 tokens x 128 latent columns
constexpr int kNKpe = 3;                     // ring of 8 KB slots: 64 tokens x 64 rope columns
constexpr int kPairBytes = 16384;
constexpr int kSubBytes = 8192;              // one 64x64 bf16 swizzled box
constexpr int kQChunkBytes = kQRows * 128;   // 16 rows x 128 B
constexpr int kQBytes = 9 * kQChunkBytes;    // 18 KB
constexpr int kPBytes = kHeads * 128;        // 16 heads x 64 tokens bf16
constexpr int kTmemCols = 128;               // S: 2 x 16 cols, O: 4 x 16 cols
constexpr int kTmemS = 0;
constexpr int kTmemO = 32;

constexpr uint32_t kIdescQK = idesc_bf16_f32(64, 16, 0, 0);   // A = C tile (K-major), B = Qa (K-major)
constexpr uint32_t kIdescPV = idesc_bf16_f32(128, 16, 1, 0);  // A = C tile (MN-major), B = P (K-major)

struct K2Smem {
    uint64_t pair_full[kNPair], pair_empty[kNPair];
    uint64_t kpe_full[kNKpe], kpe_empty[kNKpe];
    uint64_t q_full, q_empty;
    uint64_t s_full[2], p_full[2], pv_done[2];
    uint64_t o_empty, teardown;
    uint32_t tmem_base;
    int abort;
    float red[2][4][16];
    float lred[4][16];
};

constexpr int kOffPair = 0;
constexpr int kOffKpe = kOffPair + kNPair * kPairBytes;
constexpr int kOffQ = kOffKpe + kNKpe * kSubBytes;
constexpr int kOffP = kOffQ + kQBytes;
constexpr int kOffMisc = kOffP + 2 * kPBytes;
constexpr int kK2SmemBytes = kOffMisc + (int)sizeof(K2Smem) + 1024;  // + alignment slack

// Walks the tiles [u_begin, u_end) of one CTA in order, tracking the request
// and the segment (run of tiles of one request). All roles walk it alike.
struct TileCursor {
    const int32_t* cum;
    const int32_t* seq_lens;
    int batch;
    int64_t u, u_begin, u_end;
    int b;
    int64_t cb0, cb1;  // cum[b], cum[b+1]
    int seg;

    __device__ void init(const int32_t* cum_, const int32_t* sl, int B, int64_t ub, int64_t ue) {
        cum = cum_; seq_lens = sl; batch = B; u = ub; u_begin = ub; u_end = ue; seg = 0;
        // largest b with cum[b] <= u (upper_bound - 1); skips empty requests
        int lo = 0, hi = B;  // cum[B] > u
        while (hi - lo > 1) {
            const int mid = (lo + hi) >> 1;
            if (cum[mid] <= u) lo = mid; else hi = mid;
        }
        b = lo; cb0 = cum[b]; cb1 = cum[b + 1];
    }
    __device__ bool valid() const { return u < u_end; }
    __device__ int page_index() const { return (int)(u - cb0); }
    __device__ int tokens() const {  // valid tokens in this 64-token tile
        const int L = seq_lens[b] + 1;
        return min(kPage, L - page_index() * kPage);
    }
    __device__ bool first() const { return u == u_begin || u == cb0; }
    __device__ bool last() const { return u == u_end - 1 || u == cb1 - 1; }
    __device__ void next() {
        ++u;
        if (u < u_end && u >= cb1) {
            ++seg;
            do { ++b; cb0 = cb1; cb1 = cum[b + 1]; } while (u >= cb1);
        }
    }
};

__device__ __forceinline__ uint32_t tmem_lane_addr(uint32_t base, int sp, int col) {
    return base + ((uint32_t)(32 * sp) << 16) + (uint32_t)col;
}

// Transposed butterfly over 16 values in lanes 0..15 of a warp (lanes 16..31
// reduce among themselves): afterwards lane i (< 16) holds the reduction of
// value (i & 15) over lanes 0..15. 15 shuffles instead of 64.
template <bool kMax>
__device__ __forceinline__ float warp_reduce16_transposed(const float (&v)[16], int lane) {
    auto op = [](float a, float b) { return kMax ? fmaxf(a, b) : a + b; };
    float r8[8], r4[4], r2[2];
    const bool u8 = lane & 8, u4 = lane & 4, u2 = lane & 2, u1 = lane & 1;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        const float send = u8 ? v[j] : v[j + 8];
        const float keep = u8 ? v[j + 8] : v[j];
        r8[j] = op(keep, __shfl_xor_sync(0xffffffffu, send, 8));
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const float send = u4 ? r8[j] : r8[j + 4];
        const float keep = u4 ? r8[j + 4] : r8[j];
        r4[j] = op(keep, __shfl_xor_sync(0xffffffffu, send, 4));
    }
#pragma unroll
    for (int j = 0; j < 2; ++j) {
        const float send = u2 ? r4[j] : r4[j + 2];
        const float keep = u2 ? r4[j + 2] : r4[j];
        r2[j] = op(keep, __shfl_xor_sync(0xffffffffu, send, 2));
    }
    const float send = u1 ? r2[0] : r2[1];
    const float keep = u1 ? r2[1] : r2[0];
    return op(keep, __shfl_xor_sync(0xffffffffu, send, 1));
}

// Wait that ignores the abort flag (used only to drain in-flight copies and
// MMAs before the CTA exits); still bounded in time.
__device__ __forceinline__ void mbar_drain(uint64_t* bar, uint32_t parity, int32_t* err) {
    int dummy = 0;
    mbar_wait(bar, parity, &dummy, err);
}

__global__ void __launch_bounds__(kK2Threads, 1)
    k2_attention_tc(const MlaDecodeParams p, const __grid_constant__ CUtensorMap tmap_kv,
                    const __grid_constant__ CUtensorMap tmap_q, float scale_log2) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    K2Smem& S = *reinterpret_cast<K2Smem*>(smem + kOffMisc);
    uint8_t* pair_s = smem + kOffPair;
    uint8_t* kpe_s = smem + kOffKpe;
    uint8_t* q_s = smem + kOffQ;
    uint8_t* p_s = smem + kOffP;

    const WsLayout ws = ws_layout(p.batch, p.num_ctas);
    char* wsb = reinterpret_cast<char*>(p.workspace);
    const int32_t* cum = reinterpret_cast<const int32_t*>(wsb + ws.tiles_cum);
    float* part_ml = reinterpret_cast<float*>(wsb + ws.part_ml);
    float* part_acc = reinterpret_cast<float*>(wsb + ws.part_acc);

    const int64_t U = cum[p.batch];
    const int G = (int)(U < (int64_t)p.num_ctas ? U : (int64_t)p.num_ctas);
    const int c = blockIdx.x;
    if (c >= G) return;  // uniform per CTA: no work, nothing allocated
    const int64_t u_begin = plan_begin(c, U, G), u_end = plan_begin(c + 1, U, G);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        for (int i = 0; i < kNPair; ++i) { mbar_init(&S.pair_full[i], 1); mbar_init(&S.pair_empty[i], 1); }
        for (int i = 0; i < kNKpe; ++i) { mbar_init(&S.kpe_full[i], 1); mbar_init(&S.kpe_empty[i], 1); }
        mbar_init(&S.q_full, 1); mbar_init(&S.q_empty, 1);
        for (int i = 0; i < 2; ++i) {
            mbar_init(&S.s_full[i], 1); mbar_init(&S.p_full[i], 128); mbar_init(&S.pv_done[i], 1);
        }
        mbar_init(&S.o_empty, 128); mbar_init(&S.teardown, 1);
        S.abort = 0;
        fence_mbar_init();
    }
    if (warp == 1) { tmem_alloc(&S.tmem_base, kTmemCols); tmem_relinquish(); }
    if (warp == 0 && lane == 0) { prefetch_tmap(&tmap_kv); prefetch_tmap(&tmap_q); }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = S.tmem_base;
    volatile int* abort = &S.abort;

    TileCursor cur;
    cur.init(cum, p.seq_lens, p.batch, u_begin, u_end);

    if (warp == 0) {
        // ------------------------------------------------------------ producer
        if (lane == 0) {
            uint32_t pair_fill = 0, kpe_fill = 0;
            int q_fill = 0;
            bool ok = true;
            for (; cur.valid() && ok; cur.next()) {
                if (cur.first()) {
                    if (q_fill > 0 && !(ok = mbar_wait(&S.q_empty, (q_fill - 1) & 1, abort, p.error_word))) break;
                    mbar_arrive_expect_tx(&S.q_full, kQBytes);
                    for (int ch = 0; ch < 9; ++ch)
                        tma_load_2d(q_s + ch * kQChunkBytes, &tmap_q, &S.q_full, 64 * ch, cur.b * kQRows,
                                    kCacheEvictLast);
                    ++q_fill;
                }
                int page = p.block_table[(int64_t)cur.b * p.max_blocks + cur.page_index()];
                if (page < 0 || page >= p.n_pages) { record_error(p.error_word, MLA_DEV_BAD_PAGE); page = 0; }
                const int row = page * kPage;
                for (int j = 0; j < 4; ++j) {
                    const uint32_t slot = pair_fill % kNPair, n = pair_fill / kNPair;
                    if (n > 0 && !(ok = mbar_wait(&S.pair_empty[slot], (n - 1) & 1, abort, p.error_word))) break;
                    mbar_arrive_expect_tx(&S.pair_full[slot], kPairBytes);
                    uint8_t* dst = pair_s + slot * kPairBytes;
                    tma_load_2d(dst, &tmap_kv, &S.pair_full[slot], 128 * j, row, kCacheEvictFirst);
                    tma_load_2d(dst + kSubBytes, &tmap_kv, &S.pair_full[slot], 128 * j + 64, row, kCacheEvictFirst);
                    ++pair_fill;
                }
                if (!ok) break;
                {
                    const uint32_t slot = kpe_fill % kNKpe, n = kpe_fill / kNKpe;
                    if (n > 0 && !(ok = mbar_wait(&S.kpe_empty[slot], (n - 1) & 1, abort, p.error_word))) break;
                    mbar_arrive_expect_tx(&S.kpe_full[slot], kSubBytes);
                    tma_load_2d(kpe_s + slot * kSubBytes, &tmap_kv, &S.kpe_full[slot], kLora, row, kCacheEvictFirst);
                    ++kpe_fill;
                }
            }
            // Drain: every issued copy must land before the CTA's shared memory is released.
            for (uint32_t s = 0; s < kNPair; ++s) {
                const uint32_t fills = pair_fill / kNPair + (s < pair_fill % kNPair ? 1u : 0u);
                if (fills) mbar_drain(&S.pair_full[s], (fills - 1) & 1, p.error_word);
            }
            for (uint32_t s = 0; s < kNKpe; ++s) {
                const uint32_t fills = kpe_fill / kNKpe + (s < kpe_fill % kNKpe ? 1u : 0u);
                if (fills) mbar_drain(&S.kpe_full[s], (fills - 1) & 1, p.error_word);
            }
            if (q_fill) mbar_drain(&S.q_full, (q_fill - 1) & 1, p.error_word);
        }
    } else if (warp == 1) {
        // ------------------------------------------------------------ MMA issuer
        if (lane == 0) {
            const uint32_t q_addr = smem_u32(q_s), p_addr = smem_u32(p_s);
            const uint32_t pair_addr = smem_u32(pair_s), kpe_addr = smem_u32(kpe_s);
            bool ok = true;
            int i = 0;
            bool prev_first = false;  // segment flags of tile i-1 (for its PV)
            int prev_seg = 0;
            auto do_pv = [&](int t, bool first, int seg) -> bool {
                if (!mbar_wait(&S.p_full[t & 1], (t >> 1) & 1, abort, p.error_word)) return false;
                tc_fence_after();
                if (first && seg > 0) {
                    if (!mbar_wait(&S.o_empty, (seg - 1) & 1, abort, p.error_word)) return false;
                    tc_fence_after();
                }
                for (int j = 0; j < 4; ++j) {
                    const uint32_t slot = (uint32_t)(4 * t + j) % kNPair;
                    const uint32_t a0 = pair_addr + slot * kPairBytes;
#pragma unroll
                    for (int ks = 0; ks < 4; ++ks) {
                        const uint64_t ad = smem_desc_sw128(a0 + ks * 2048, kSubBytes, 1024);
                        const uint64_t bd = smem_desc_sw128(p_addr + (t & 1) * kPBytes + ks * 32, 16, 1024);
                        tc_mma_f16(tmem + kTmemO + 16 * j, ad, bd, kIdescPV, (first && ks == 0) ? 0u : 1u);
                    }
                    tc_commit(&S.pair_empty[slot]);
                }
                tc_commit(&S.pv_done[t & 1]);
                return true;
            };
            for (; cur.valid(); cur.next(), ++i) {
                if (cur.first()) {
                    if (!(ok = mbar_wait(&S.q_full, cur.seg & 1, abort, p.error_word))) break;
                    tc_fence_after();
                }
                const uint32_t d_s = tmem + kTmemS + 16 * (i & 1);
                for (int ch = 0; ch < 9 && ok; ++ch) {
                    uint32_t a_addr;
                    if (ch < 8) {
                        const uint32_t fill = (uint32_t)(4 * i + ch / 2), slot = fill % kNPair;
                        if ((ch & 1) == 0) {
                            if (!(ok = mbar_wait(&S.pair_full[slot], (fill / kNPair) & 1, abort, p.error_word))) break;
                            tc_fence_after();
                        }
                        a_addr = pair_addr + slot * kPairBytes + (ch & 1) * kSubBytes;
                    } else {
                        const uint32_t slot = (uint32_t)i % kNKpe;
                        if (!(ok = mbar_wait(&S.kpe_full[slot], ((uint32_t)i / kNKpe) & 1, abort, p.error_word))) break;
                        tc_fence_after();
                        a_addr = kpe_addr + slot * kSubBytes;
                    }
#pragma unroll
                    for (int kk = 0; kk < 4; ++kk) {
                        const uint64_t ad = smem_desc_sw128(a_addr + kk * 32, 16, 1024);
                        const uint64_t bd = smem_desc_sw128(q_addr + ch * kQChunkBytes + kk * 32, 16, 1024);
                        tc_mma_f16(d_s, ad, bd, kIdescQK, (ch | kk) ? 1u : 0u);
                    }
                }
                if (!ok) break;
                tc_commit(&S.s_full[i & 1]);
                tc_commit(&S.kpe_empty[(uint32_t)i % kNKpe]);
                if (cur.last()) tc_commit(&S.q_empty);
                if (i > 0 && !(ok = do_pv(i - 1, prev_first, prev_seg))) break;
                prev_first = cur.first();
                prev_seg = cur.seg;
            }
            if (ok && i > 0) do_pv(i - 1, prev_first, prev_seg);
            // Drain all issued MMAs before TMEM is freed.
            tc_commit(&S.teardown);
            mbar_drain(&S.teardown, 0, p.error_word);
        }
    } else {
        // ------------------------------------------------------------ softmax + epilogue
        const int sp = warp & 3;            // TMEM subpartition of this warp
        const int tok = 16 * sp + lane;     // token of this lane in the 64-token tile (lane < 16)
        const int wg_tid = threadIdx.x - 64;
        float m_run[16], l_thr[16];
#pragma unroll
        for (int h = 0; h < 16; ++h) { m_run[h] = -INFINITY; l_thr[h] = 0.f; }
        int i = 0;
        for (; cur.valid(); cur.next(), ++i) {
            const bool first = cur.first(), last = cur.last();
            const int valid = cur.tokens();
            if (first) {
#pragma unroll
                for (int h = 0; h < 16; ++h) { m_run[h] = -INFINITY; l_thr[h] = 0.f; }
            }
            if (!mbar_wait(&S.s_full[i & 1], (i >> 1) & 1, abort, p.error_word)) break;
            tc_fence_after();
            __syncwarp();
            float s[16];
            tmem_ld16(tmem_lane_addr(tmem, sp, kTmemS + 16 * (i & 1)), s);
            tmem_wait_ld();
            const bool ok_tok = lane < 16 && tok < valid;
#pragma unroll
            for (int h = 0; h < 16; ++h) s[h] = ok_tok ? s[h] * scale_log2 : -INFINITY;

            const float wmax = warp_reduce16_transposed<true>(s, lane);
            if (lane < 16) S.red[i & 1][sp][lane] = wmax;
            named_bar_sync(1, 128);
            float mt[16];
#pragma unroll
            for (int h = 0; h < 16; ++h)
                mt[h] = fmaxf(fmaxf(S.red[i & 1][0][h], S.red[i & 1][1][h]), fmaxf(S.red[i & 1][2][h], S.red[i & 1][3][h]));

            if (first) {
#pragma unroll
                for (int h = 0; h < 16; ++h) m_run[h] = mt[h];
            } else {
                // Lazy rescale: keep the running max unless a head's tile max
                // exceeds it by more than 2^8; exps stay <= 256 in between.
                bool need = false;
#pragma unroll
                for (int h = 0; h < 16; ++h) need |= mt[h] > m_run[h] + 8.f;
                if (need) {
                    float f[16];
#pragma unroll
                    for (int h = 0; h < 16; ++h) {
                        const float mn = fmaxf(m_run[h], mt[h]);
                        f[h] = fast_exp2(m_run[h] - mn);
                        m_run[h] = mn;
                        l_thr[h] *= f[h];
                    }
                    if (!mbar_wait(&S.pv_done[(i - 1) & 1], ((i - 1) >> 1) & 1, abort, p.error_word)) break;
                    tc_fence_after();
                    __syncwarp();
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        float o[16];
                        const uint32_t ta = tmem_lane_addr(tmem, sp, kTmemO + 16 * j);
                        tmem_ld16(ta, o);
                        tmem_wait_ld();
#pragma unroll
                        for (int h = 0; h < 16; ++h) o[h] *= f[h];
                        tmem_st16(ta, o);
                    }
                    tmem_wait_st();
                }
            }
            float pr[16];
#pragma unroll
            for (int h = 0; h < 16; ++h) {
                const float e = ok_tok ? bf16_round(fast_exp2(s[h] - m_run[h])) : 0.f;
                pr[h] = e;
                l_thr[h] += e;
            }
            // P buffer (i & 1) is free once the output MMA of tile i-2 is done.
            if (i >= 2 && !mbar_wait(&S.pv_done[i & 1], ((i - 2) >> 1) & 1, abort, p.error_word)) break;
            if (lane < 16) {
                uint8_t* pb = p_s + (i & 1) * kPBytes;
#pragma unroll
                for (int h = 0; h < 16; ++h) {
                    const int off = (h >> 3) * 1024 + (h & 7) * 128 + ((((tok >> 3) ^ (h & 7))) << 4) + (tok & 7) * 2;
                    *reinterpret_cast<__nv_bfloat16*>(pb + off) = __float2bfloat16_rn(pr[h]);
                }
            }
            if (valid < kPage) {
                // Rows past the sequence end are masked in P; zero them in the
                // C tile too so that 0 * (stale or non-finite bits) cannot
                // reach the output MMA.
                bool okw = true;
                for (int j = 0; j < 4 && okw; ++j) {
                    const uint32_t fill = (uint32_t)(4 * i + j);
                    okw = mbar_wait(&S.pair_full[fill % kNPair], (fill / kNPair) & 1, abort, p.error_word);
                }
                if (!okw) break;
                const int nrows = kPage - valid;
                const int per_sub = nrows * 8;
                for (int idx = wg_tid; idx < 8 * per_sub; idx += 128) {
                    const int sub = idx / per_sub, rem = idx % per_sub;
                    const int r = valid + rem / 8, q16 = rem % 8;
                    const uint32_t slot = (uint32_t)(4 * i + sub / 2) % kNPair;
                    uint8_t* dst = pair_s + slot * kPairBytes + (sub & 1) * kSubBytes + r * 128 + q16 * 16;
                    *reinterpret_cast<uint4*>(dst) = make_uint4(0, 0, 0, 0);
                }
            }
            fence_proxy_async_smem();
            tc_fence_before();
            mbar_arrive(&S.p_full[i & 1]);

            if (last) {
                if (!mbar_wait(&S.pv_done[i & 1], (i >> 1) & 1, abort, p.error_word)) break;
                tc_fence_after();
                const float lsum = warp_reduce16_transposed<false>(l_thr, lane);
                if (lane < 16) S.lred[sp][lane] = lsum;
                named_bar_sync(1, 128);
                const int slot = c + cur.b;
                if (sp == 0 && lane < 16) {
                    float m_h = 0.f;
#pragma unroll
                    for (int h = 0; h < 16; ++h) if (h == lane) m_h = m_run[h];
                    const float l_h = (S.lred[0][lane] + S.lred[1][lane]) + (S.lred[2][lane] + S.lred[3][lane]);
                    part_ml[((int64_t)slot * kHeads + lane) * 2 + 0] = m_h;
                    part_ml[((int64_t)slot * kHeads + lane) * 2 + 1] = l_h;
                }
                float* acc = part_acc + (int64_t)slot * kHeads * kLora;
                __syncwarp();
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    float o[16];
                    tmem_ld16(tmem_lane_addr(tmem, sp, kTmemO + 16 * j), o);
                    tmem_wait_ld();
#pragma unroll
                    for (int h = 0; h < 16; ++h) acc[h * kLora + 128 * j + 32 * sp + lane] = o[h];
                }
                tc_fence_before();
                mbar_arrive(&S.o_empty);
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        __syncwarp();
        tc_fence_after();
        tmem_dealloc(tmem, kTmemCols);
    }
}

// ---------------------------------------------------------------------------
// Checker kernel: the same plan and partial layout on CUDA cores in fp32,
// with exact (non-lazy) online-softmax rescaling and fp32 probabilities.
// It exists to cross-check the tensor-core kernel on the GPU.
// ---------------------------------------------------------------------------
constexpr int kCkThreads = 256;

__global__ void __launch_bounds__(kCkThreads)
    k2_attention_check(const MlaDecodeParams p, float scale_log2) {
    extern __shared__ uint8_t smem_raw[];
    float* qf = reinterpret_cast<float*>(smem_raw);                       // [16][576]
    __nv_bfloat16* tile = reinterpret_cast<__nv_bfloat16*>(qf + kHeads * kRow);  // [64][576]
    float* sc = reinterpret_cast<float*>(tile + kPage * kRow);            // [16][64]

    const WsLayout ws = ws_layout(p.batch, p.num_ctas);
    char* wsb = reinterpret_cast<char*>(p.workspace);
    const int32_t* cum = reinterpret_cast<const int32_t*>(wsb + ws.tiles_cum);
    const __nv_bfloat16* qa = reinterpret_cast<const __nv_bfloat16*>(wsb + ws.qa);
    float* part_ml = reinterpret_cast<float*>(wsb + ws.part_ml);
    float* part_acc = reinterpret_cast<float*>(wsb + ws.part_acc);
    const __nv_bfloat16* cache = reinterpret_cast<const __nv_bfloat16*>(p.kv_cache);

    const int64_t U = cum[p.batch];
    const int G = (int)(U < (int64_t)p.num_ctas ? U : (int64_t)p.num_ctas);
    const int c = blockIdx.x;
    if (c >= G) return;
    TileCursor cur;
    cur.init(cum, p.seq_lens, p.batch, plan_begin(c, U, G), plan_begin(c + 1, U, G));

    const int h = threadIdx.x >> 4, part = threadIdx.x & 15;  // head, 32-column slice of the latent
    float acc[32];
    float m_run = -INFINITY, l_run = 0.f;
    for (; cur.valid(); cur.next()) {
        if (cur.first()) {
            __syncthreads();
            for (int i = threadIdx.x; i < kHeads * kRow; i += kCkThreads)
                qf[i] = __bfloat162float(qa[(int64_t)cur.b * kQRows * kRow + i]);
#pragma unroll
            for (int k = 0; k < 32; ++k) acc[k] = 0.f;
            m_run = -INFINITY; l_run = 0.f;
        }
        int page = p.block_table[(int64_t)cur.b * p.max_blocks + cur.page_index()];
        if (page < 0 || page >= p.n_pages) { record_error(p.error_word, MLA_DEV_BAD_PAGE); page = 0; }
        const int valid = cur.tokens();
        __syncthreads();
        {
            const uint4* src = reinterpret_cast<const uint4*>(cache + (int64_t)page * kPage * kRow);
            uint4* dst = reinterpret_cast<uint4*>(tile);
            for (int i = threadIdx.x; i < kPage * kRow / 8; i += kCkThreads) {
                const int r = i / (kRow / 8);
                dst[i] = r < valid ? src[i] : make_uint4(0, 0, 0, 0);
            }
        }
        __syncthreads();
        for (int t = part; t < kPage; t += 16) {
            float s = 0.f;
            for (int k = 0; k < kRow; ++k) s = fmaf(qf[h * kRow + k], __bfloat162float(tile[t * kRow + k]), s);
            sc[h * kPage + t] = t < valid ? s * scale_log2 : -INFINITY;
        }
        __syncwarp();
        float mx = -INFINITY;
        for (int t = part; t < kPage; t += 16) mx = fmaxf(mx, sc[h * kPage + t]);
#pragma unroll
        for (int o = 8; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
        const float m_new = fmaxf(m_run, mx);
        const float f = exp2f(m_run - m_new);
        float ls = 0.f;
        for (int t = part; t < kPage; t += 16) {
            const float e = t < valid ? exp2f(sc[h * kPage + t] - m_new) : 0.f;
            sc[h * kPage + t] = e;
            ls += e;
        }
#pragma unroll
        for (int o = 8; o; o >>= 1) ls += __shfl_xor_sync(0xffffffffu, ls, o);
        l_run = l_run * f + ls;
        m_run = m_new;
        __syncwarp();
#pragma unroll
        for (int k = 0; k < 32; ++k) acc[k] *= f;
        for (int t = 0; t < valid; ++t) {
            const float pt = sc[h * kPage + t];
#pragma unroll
            for (int k = 0; k < 32; ++k) acc[k] = fmaf(pt, __bfloat162float(tile[t * kRow + 32 * part + k]), acc[k]);
        }
        if (cur.last()) {
            const int slot = c + cur.b;
            if (part == 0) {
                part_ml[((int64_t)slot * kHeads + h) * 2 + 0] = m_run;
                part_ml[((int64_t)slot * kHeads + h) * 2 + 1] = l_run;
            }
            float* dst = part_acc + ((int64_t)slot * kHeads + h) * kLora + 32 * part;
#pragma unroll
            for (int k = 0; k < 32; ++k) dst[k] = acc[k];
        }
    }
}

constexpr int kCkSmemBytes = kHeads * kRow * 4 + kPage * kRow * 2 + kHeads * kPage * 4;

// ---------------------------------------------------------------------------
// Host-side launch helpers (called from mla_abi.cu).
// ---------------------------------------------------------------------------
int k2_smem_bytes() { return kK2SmemBytes; }
int k2_check_smem_bytes() { return kCkSmemBytes; }

cudaError_t k2_configure() {
    cudaError_t e = cudaFuncSetAttribute(k2_attention_tc, cudaFuncAttributeMaxDynamicSharedMemorySize, kK2SmemBytes);
    if (e != cudaSuccess) return e;
    return cudaFuncSetAttribute(k2_attention_check, cudaFuncAttributeMaxDynamicSharedMemorySize, kCkSmemBytes);
}

cudaError_t launch_attention_tc(const MlaDecodeParams& p, const CUtensorMap& tmap_kv, const CUtensorMap& tmap_q,
                                float scale_log2, cudaStream_t stream) {
    k2_attention_tc<<<p.num_ctas, kK2Threads, kK2SmemBytes, stream>>>(p, tmap_kv, tmap_q, scale_log2);
    return cudaGetLastError();
}

cudaError_t launch_attention_check(const MlaDecodeParams& p, float scale_log2, cudaStream_t stream) {
    k2_attention_check<<<p.num_ctas, kCkThreads, kCkSmemBytes, stream>>>(p, scale_log2);
    return cudaGetLastError();
}

}  // namespace mla
