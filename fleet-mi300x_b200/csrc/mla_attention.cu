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
#include "mla_tiles.cuh"

namespace mla {

constexpr int kK2Threads = 192;
constexpr int kNTile = 2;                    // ring of whole-page tiles (one TMA request each)
constexpr int kChunkBytes = 8192;            // one [64 tokens x 64 columns] bf16 swizzled block
constexpr int kTileBytes = 9 * kChunkBytes;  // a page: 9 column blocks (8 of c_kv, 1 of k_pe)
constexpr int kQChunkBytes = kQRows * 128;   // 16 rows x 128 B
constexpr int kQBytes = 9 * kQChunkBytes;    // 18 KB
constexpr int kNQ = 2;                       // absorbed-query buffers (one per segment in flight)
constexpr int kPBytes = kHeads * 128;        // 16 heads x 64 tokens bf16
// TMEM columns: S (scores) double-buffered, each buffer 4 partial sums x 16
// heads (independent accumulation chains, summed by the softmax); O: 4 latent
// blocks x 16 heads.
constexpr int kSParts = 4;
constexpr int kTmemCols = 256;
constexpr int kTmemS = 0;                     // + 64 * buffer + 16 * part
constexpr int kTmemO = 2 * kSParts * 16;      // 128

#ifdef MLA_TRACE
__device__ long long g_mla_trace[kTraceCtas * kTraceTiles * kTraceEvents];
#endif

constexpr uint32_t kIdescQK = idesc_bf16_f32(64, 16, 0, 0);   // A = C tile (K-major), B = Qa (K-major)
constexpr uint32_t kIdescPV = idesc_bf16_f32(128, 16, 1, 0);  // A = C tile (MN-major), B = P (K-major)

struct K2Smem {
    uint64_t tile_full[kNTile], tile_empty[kNTile];
    uint64_t q_full[kNQ], q_empty[kNQ];
    uint64_t s_full[2], p_full[2], pv_done[2];
    uint64_t o_empty, teardown;
    uint32_t tmem_base;
    int abort;
    float red[2][4][16];
    float lred[4][16];
};

constexpr int kOffTile = 0;
constexpr int kOffQ = kOffTile + kNTile * kTileBytes;
constexpr int kOffP = kOffQ + kNQ * kQBytes;
constexpr int kOffMisc = kOffP + 2 * kPBytes;
constexpr int kK2SmemBytes = kOffMisc + (int)sizeof(K2Smem) + 1024;  // + alignment slack
static_assert(kK2SmemBytes <= 232448, "K2 shared memory exceeds 227 KB");

__global__ void __launch_bounds__(kK2Threads, 1)
    k2_attention_tc(const MlaDecodeParams p, const __grid_constant__ CUtensorMap tmap_kv,
                    const __grid_constant__ CUtensorMap tmap_q, float scale_log2) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    K2Smem& S = *reinterpret_cast<K2Smem*>(smem + kOffMisc);
    uint8_t* tile_s = smem + kOffTile;
    uint8_t* q_s = smem + kOffQ;
    uint8_t* p_s = smem + kOffP;

    const WsLayout ws = ws_layout(p);
    char* wsb = reinterpret_cast<char*>(p.workspace);
    const int32_t* cum = reinterpret_cast<const int32_t*>(wsb + ws.tiles_cum);
    float* part_ml = reinterpret_cast<float*>(wsb + ws.part_ml);
    float* part_acc = reinterpret_cast<float*>(wsb + ws.part_acc);

    pdl_trigger();
    pdl_wait();  // the plan, absorbed queries and new rows come from K1
    const int64_t U = cum[p.batch];
    const int G = (int)(U < (int64_t)p.num_ctas ? U : (int64_t)p.num_ctas);
    const int c = blockIdx.x;
    if (c >= G) return;  // uniform per CTA: no work, nothing allocated
    const int64_t u_begin = plan_begin(c, U, G), u_end = plan_begin(c + 1, U, G);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        for (int i = 0; i < kNTile; ++i) { mbar_init(&S.tile_full[i], 1); mbar_init(&S.tile_empty[i], 1); }
        for (int i = 0; i < kNQ; ++i) { mbar_init(&S.q_full[i], 1); mbar_init(&S.q_empty[i], 1); }
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
    cur.init(cum, p.seq_lens, p.batch, u_begin, u_end, new_row_count(p));

    if (warp == 0) {
        // ------------------------------------------------------------ producer
        // One TMA request per 64-token page (4-D box {64, 64, 9, 1}: 72 KB,
        // landing as 9 swizzled [64 x 64] column blocks), and one per
        // segment for the absorbed query (3-D box {64, 16, 9}: 18 KB).
        if (lane == 0) {
            uint32_t t = 0;
            int q_fill = 0;
            bool ok = true;
            for (; cur.valid() && ok; cur.next(), ++t) {
                MLA_STAMP((int)t, 0);
                if (cur.first()) {
                    const int qs = q_fill % kNQ, n = q_fill / kNQ;
                    if (n > 0 && !(ok = mbar_wait(&S.q_empty[qs], (n - 1) & 1, abort, err_sink(p)))) break;
                    mbar_arrive_expect_tx(&S.q_full[qs], kQBytes);
                    tma_load_3d(q_s + qs * kQBytes, &tmap_q, &S.q_full[qs], 0, cur.b * kQRows, 0, kCacheEvictLast);
                    ++q_fill;
                }
                int page = p.block_table[(int64_t)cur.b * p.max_blocks + cur.page_index()];
                if (page < 0 || page >= p.n_pages) { record_error(err_sink(p), MLA_DEV_BAD_PAGE); page = 0; }
                const uint32_t slot = t % kNTile, n = t / kNTile;
                if (n > 0 && !(ok = mbar_wait(&S.tile_empty[slot], (n - 1) & 1, abort, err_sink(p)))) break;
                mbar_arrive_expect_tx(&S.tile_full[slot], kTileBytes);
                tma_load_4d(tile_s + slot * kTileBytes, &tmap_kv, &S.tile_full[slot], 0, 0, 0, page, kCacheEvictFirst);
                MLA_STAMP((int)t, 1);
            }
            // Drain: every issued copy must land before the CTA's shared memory is released.
            for (uint32_t sl = 0; sl < kNTile; ++sl) {
                const uint32_t fills = t / kNTile + (sl < t % kNTile ? 1u : 0u);
                if (fills) mbar_drain(&S.tile_full[sl], (fills - 1) & 1, err_sink(p));
            }
            for (int qs = 0; qs < kNQ; ++qs) {
                const int fills = q_fill / kNQ + (qs < q_fill % kNQ ? 1 : 0);
                if (fills) mbar_drain(&S.q_full[qs], (fills - 1) & 1, err_sink(p));
            }
        }
    } else if (warp == 1) {
        // ------------------------------------------------------------ MMA issuer
        // Event-driven: polls (non-blocking) for the next output MMA (P of the
        // oldest tile ready) and the next score MMA (its page landed), output
        // first. S is double-buffered, so the score MMA of tile j may run
        // ahead of the output MMA of tile j-2 only.
        if (lane == 0) {
            const uint32_t q_addr = smem_u32(q_s), p_addr = smem_u32(p_s), tile_addr = smem_u32(tile_s);
            // Descriptors differ only in the start-address field: build the
            // constant high part once and add (address >> 4).
            const uint64_t dK = smem_desc_sw128(0, 16, 1024);          // K-major, 8-row groups 1024 B apart
            const uint64_t dMN = smem_desc_sw128(0, kChunkBytes, 1024);  // MN-major, 64-column blocks 8 KB apart
            const int n_tiles = (int)(u_end - u_begin);
            struct TileInfo { bool first, last; int seg; };
            TileInfo info[4] = {};  // entry t & 3 is written by the score step of tile t before P of t exists
            int qk_j = 0, pv_next = 0;

            auto pv_step = [&]() -> bool {
                if (!mbar_test_wait(&S.p_full[pv_next & 1], (pv_next >> 1) & 1)) return false;
                const TileInfo ti = info[pv_next & 3];
                if (ti.first && ti.seg > 0 && !mbar_test_wait(&S.o_empty, (ti.seg - 1) & 1)) return false;
                tc_fence_after();
                const int t = pv_next;
                MLA_STAMP(t, 4);
                const uint32_t a0 = tile_addr + (uint32_t)(t % kNTile) * kTileBytes;
                const uint32_t b0 = p_addr + (t & 1) * kPBytes;
                // k-step-major: consecutive MMAs feed the 4 independent output
                // blocks, so no MMA waits on the one just issued.
#pragma unroll
                for (int ks = 0; ks < 4; ++ks) {
                    const uint64_t bd = dK + ((b0 + ks * 32) >> 4);
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        const uint64_t ad = dMN + ((a0 + j * 2 * kChunkBytes + ks * 2048) >> 4);
                        tc_mma_f16(tmem + kTmemO + 16 * j, ad, bd, kIdescPV, (ti.first && ks == 0) ? 0u : 1u);
                    }
                }
                tc_commit(&S.tile_empty[t % kNTile]);
                tc_commit(&S.pv_done[t & 1]);
                MLA_STAMP(t, 5);
                ++pv_next;
                return true;
            };

            auto qk_step = [&]() -> bool {
                const bool first = cur.first();
                const int qs = cur.seg % kNQ;
                if (first && !mbar_test_wait(&S.q_full[qs], (cur.seg / kNQ) & 1)) return false;
                const uint32_t slot = (uint32_t)qk_j % kNTile;
                if (!mbar_test_wait(&S.tile_full[slot], ((uint32_t)qk_j / kNTile) & 1)) return false;
                tc_fence_after();
                MLA_STAMP(qk_j, 2);
                info[qk_j & 3] = TileInfo{first, cur.last(), cur.seg};
                const uint32_t a0 = tile_addr + slot * kTileBytes;
                const uint32_t b0 = q_addr + qs * kQBytes;
                // Sub-step kk of every 64-column block accumulates into its own
                // partial S_kk: 4 independent chains of 9 MMAs, interleaved.
                const uint32_t d_s = tmem + kTmemS + 64 * (qk_j & 1);
#pragma unroll
                for (int ch = 0; ch < 9; ++ch) {
#pragma unroll
                    for (int kk = 0; kk < kSParts; ++kk) {
                        const uint64_t ad = dK + ((a0 + ch * kChunkBytes + kk * 32) >> 4);
                        const uint64_t bd = dK + ((b0 + ch * kQChunkBytes + kk * 32) >> 4);
                        tc_mma_f16(d_s + 16 * kk, ad, bd, kIdescQK, ch ? 1u : 0u);
                    }
                }
                tc_commit(&S.s_full[qk_j & 1]);
                if (cur.last()) tc_commit(&S.q_empty[qs]);
                MLA_STAMP(qk_j, 3);
                ++qk_j;
                cur.next();
                return true;
            };

            uint32_t idle = 0;
            uint64_t idle_t0 = 0;
            while (pv_next < n_tiles) {
                bool prog = false;
                if (pv_next < qk_j) prog = pv_step();
                if (!prog && qk_j < n_tiles && qk_j < pv_next + 2) prog = qk_step();
                if (prog) { idle = 0; continue; }
                if ((++idle & 63) == 0) {
                    if (*abort) break;
                    const uint64_t now = globaltimer_ns();
                    if (idle == 64) {
                        idle_t0 = now;
                    } else if (now - idle_t0 > kWaitLimitNs) {
                        record_error(err_sink(p), MLA_DEV_TIMEOUT);
                        *abort = 1;
                        break;
                    }
                }
            }
            // Drain all issued MMAs before TMEM is freed.
            tc_commit(&S.teardown);
            mbar_drain(&S.teardown, 0, err_sink(p));
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
            if (!mbar_wait(&S.s_full[i & 1], (i >> 1) & 1, abort, err_sink(p))) break;
            tc_fence_after();
            __syncwarp();
            if (wg_tid == 0) MLA_STAMP(i, 6);
            float s[16];
            {
                float s1[16], s2[16], s3[16];
                const uint32_t ta = tmem_lane_addr(tmem, sp, kTmemS + 64 * (i & 1));
                tmem_ld16(ta, s);
                tmem_ld16(ta + 16, s1);
                tmem_ld16(ta + 32, s2);
                tmem_ld16(ta + 48, s3);
                tmem_wait_ld();
#pragma unroll
                for (int h = 0; h < 16; ++h) s[h] = (s[h] + s1[h]) + (s2[h] + s3[h]);
            }
            const bool ok_tok = lane < 16 && tok < valid;
#pragma unroll
            for (int h = 0; h < 16; ++h) s[h] = ok_tok ? s[h] * scale_log2 : -INFINITY;

            // Running max per head (log2 domain). First tile of a segment: the
            // exact tile max. Later tiles: lazy rescale; the running max is
            // kept unless some score exceeds it by more than 8 (exps stay
            // <= 256), which all 128 threads decide in one barrier-reduction.
            bool exchange = first;
            if (!first) {
                bool exceed = false;
#pragma unroll
                for (int h = 0; h < 16; ++h) exceed |= s[h] > m_run[h] + 8.f;
                exchange = bar_red_or(1, 128, exceed);
            }
            if (exchange) {
                const float wmax = warp_reduce16_transposed<true>(s, lane);
                if (lane < 16) S.red[i & 1][sp][lane] = wmax;
                named_bar_sync(1, 128);
                float mt[16];
#pragma unroll
                for (int h = 0; h < 16; ++h)
                    mt[h] = fmaxf(fmaxf(S.red[i & 1][0][h], S.red[i & 1][1][h]),
                                  fmaxf(S.red[i & 1][2][h], S.red[i & 1][3][h]));
                if (first) {
#pragma unroll
                    for (int h = 0; h < 16; ++h) m_run[h] = mt[h];
                } else {
                    float f[16];
#pragma unroll
                    for (int h = 0; h < 16; ++h) {
                        const float mn = fmaxf(m_run[h], mt[h]);
                        f[h] = fast_exp2(m_run[h] - mn);
                        m_run[h] = mn;
                        l_thr[h] *= f[h];
                    }
                    if (!mbar_wait(&S.pv_done[(i - 1) & 1], ((i - 1) >> 1) & 1, abort, err_sink(p))) break;
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
            if (i >= 2 && !mbar_wait(&S.pv_done[i & 1], ((i - 2) >> 1) & 1, abort, err_sink(p))) break;
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
                const uint32_t slot = (uint32_t)i % kNTile;
                if (!mbar_wait(&S.tile_full[slot], ((uint32_t)i / kNTile) & 1, abort, err_sink(p))) break;
                const int nrows = kPage - valid;
                const int per_chunk = nrows * 8;
                uint8_t* base = tile_s + slot * kTileBytes;
                for (int idx = wg_tid; idx < 8 * per_chunk; idx += 128) {
                    const int ch = idx / per_chunk, rem = idx % per_chunk;
                    const int r = valid + rem / 8, q16 = rem % 8;
                    *reinterpret_cast<uint4*>(base + ch * kChunkBytes + r * 128 + q16 * 16) = make_uint4(0, 0, 0, 0);
                }
            }
            fence_proxy_async_smem();
            tc_fence_before();
            mbar_arrive(&S.p_full[i & 1]);
            if (wg_tid == 0) MLA_STAMP(i, 7);

            if (last) {
                if (!mbar_wait(&S.pv_done[i & 1], (i >> 1) & 1, abort, err_sink(p))) break;
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

    const WsLayout ws = ws_layout(p);
    char* wsb = reinterpret_cast<char*>(p.workspace);
    const int32_t* cum = reinterpret_cast<const int32_t*>(wsb + ws.tiles_cum);
    const __nv_bfloat16* qa = reinterpret_cast<const __nv_bfloat16*>(wsb + ws.qa);
    float* part_ml = reinterpret_cast<float*>(wsb + ws.part_ml);
    float* part_acc = reinterpret_cast<float*>(wsb + ws.part_acc);
    const __nv_bfloat16* cache = reinterpret_cast<const __nv_bfloat16*>(p.kv_cache);

    pdl_trigger();
    pdl_wait();  // the plan, absorbed queries and new rows come from K1
    const int64_t U = cum[p.batch];
    const int G = (int)(U < (int64_t)p.num_ctas ? U : (int64_t)p.num_ctas);
    const int c = blockIdx.x;
    if (c >= G) return;
    TileCursor cur;
    cur.init(cum, p.seq_lens, p.batch, plan_begin(c, U, G), plan_begin(c + 1, U, G), new_row_count(p));

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
        if (page < 0 || page >= p.n_pages) { record_error(err_sink(p), MLA_DEV_BAD_PAGE); page = 0; }
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
    const cudaError_t e = launch_pdl(k2_attention_tc, dim3(p.num_ctas), dim3(kK2Threads), kK2SmemBytes, stream, p,
                                     tmap_kv, tmap_q, scale_log2);
    if (e != cudaSuccess) return e;
    return cudaGetLastError();
}

cudaError_t launch_attention_check(const MlaDecodeParams& p, float scale_log2, cudaStream_t stream) {
    const cudaError_t e = launch_pdl(k2_attention_check, dim3(p.num_ctas), dim3(kCkThreads), kCkSmemBytes, stream, p,
                                     scale_log2);
    if (e != cudaSuccess) return e;
    return cudaGetLastError();
}

}  // namespace mla

#ifdef MLA_TRACE
namespace mla {
__device__ unsigned long long g_mla_timeline[kTlKernels * kTlCtas * kTlEvents];
}  // namespace mla

// Trace build only (not part of include/mla_decode.h): copy the kernel timeline
// [5 kernels][512 CTAs][6: entry, after pdl_wait, exit (%globaltimer ns, 0 = not
// stamped), SM id + 1, mark 1, mark 2] to `host` and clear it.
extern "C" int mla_timeline_read(unsigned long long* host, uint64_t n) {
    using namespace mla;
    const uint64_t total = (uint64_t)kTlKernels * kTlCtas * kTlEvents;
    if (!host || n < total) return MLA_E_INVALID_ARG;
    if (cudaMemcpyFromSymbol(host, g_mla_timeline, total * sizeof(unsigned long long)) != cudaSuccess)
        return MLA_E_LAUNCH;
    static unsigned long long zeros[kTlKernels * kTlCtas * kTlEvents];
    if (cudaMemcpyToSymbol(g_mla_timeline, zeros, sizeof(zeros)) != cudaSuccess) return MLA_E_LAUNCH;
    return MLA_OK;
}

// Trace build only (not part of include/mla_decode.h): copy the attention
// kernel's per-tile stamps [160 CTAs][96 tiles][8 events] (SM clocks) to `host`
// and clear them.
extern "C" int mla_trace_read(long long* host, uint64_t n) {
    using namespace mla;
    const uint64_t total = (uint64_t)kTraceCtas * kTraceTiles * kTraceEvents;
    if (!host || n < total) return MLA_E_INVALID_ARG;
    if (cudaMemcpyFromSymbol(host, g_mla_trace, total * sizeof(long long)) != cudaSuccess) return MLA_E_LAUNCH;
    static long long zeros[kTraceCtas * kTraceTiles * kTraceEvents];
    if (cudaMemcpyToSymbol(g_mla_trace, zeros, sizeof(zeros)) != cudaSuccess) return MLA_E_LAUNCH;
    return MLA_OK;
}
#endif
