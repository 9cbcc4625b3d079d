// K2 (default) — split-KV absorbed-MLA attention with exactly 16 heads on the
// MMA's M dimension: mma.sync m16n8k16 (bf16 in, fp32 accumulate) fed by
// half-page TMA tiles, two independent compute groups per CTA.
//
// Why this shape: with 16 heads and one query per request the contractions
// are [16 x 576] x [576 x tokens] (scores) and [16 x tokens] x [tokens x 512]
// (output). A 5th-generation (tcgen05) MMA costs the same issue slot whatever
// its N, so at N = 16 it runs ~16x below its rate and the score contraction
// alone cannot keep up with HBM; m16n8k16 has M = 16 = heads exactly. The
// tensor-memory kernel (mla_attention.cu) stays available for comparison.
//
// Why two groups: one group's work per tile is a serial chain (scores ->
// score exchange -> softmax -> output, with group barriers), and with one
// warp per scheduler a 64-token page took ~1.5 us of it against ~1.6 us of
// HBM time per page per SM. Two groups of four warps (one warp of each on
// every scheduler) run independent chains that hide each other's latency.
// Each group is one CTA of the split-KV plan (vc = CTA + grid * group),
// with its own 2-slot ring of 32-row half pages (36 KB, one contiguous
// stretch of the page, one TMA box each), so the plan and the partial layout
// are those of num_ctas virtual CTAs and K3 is unchanged.
//
// Per group (4 warps), per half page:
//   scores    S_w = Q[:, 144w : 144w+144] C[:, 144w : 144w+144]^T for the 32
//             tokens (9 k-steps x 4 token tiles), Q fragments in registers;
//   exchange  the 4 partial S through shared memory; warp w sums the 8 tokens
//             [8w, 8w+8) and runs the softmax on them;
//   softmax   lazy rescale: the running max per head is kept unless a score
//             exceeds it by more than 2^8; probabilities are rounded to bf16 and
//             written with the running max, and one barrier-reduction both
//             publishes them and decides whether to rescale and write them again;
//   output    O_w[16 x 128] += P[16 x 32] C[:, 128w : 128w+128] (2 k-steps x
//             16 latent tiles), accumulated in registers (rescale = multiply).
// Loads: the group's leader thread issues half page j+2 into the slot of half
// page j as soon as all four warps have released it (mbarrier, bounded wait).
// Segment ends: the last half page of a request's segment requests the next
// segment's query fragments before writing its partial, so that their latency
// overlaps the partial's stores.
// The split plan's tiles are these half pages (plan_unit_rows), so a request's
// rows split between plan CTAs at 32-row granularity and a request with up to
// 32 rows in its last page loads only that half.
// Start: batches of up to 64 requests derive the split plan from the step's
// inputs before the wait on K1 and request their first half page early (except
// one holding the row K1 appends); larger batches read K1's per-CTA plan entry.
// Pairs (k2_pairs, G = num_ctas): the two groups hold adjacent plan CTAs 2k, 2k + 1;
// where their boundary falls inside a request, group 1's first partial is merged
// into group 0's last one in shared memory (slot 2k + b), so K3 folds fewer.
// Precision forms (template flags): kQLo (MLA_FLAG_QC_HILO) adds the score MMAs of
// the low half of q_c (K1's qa_lo) over the 512 latent columns; kPLo
// (MLA_FLAG_P_HILO) keeps each probability as bf16 hi + lo in two P buffers, runs
// the output MMAs on both and sums the row totals over the unrounded values.
#include <cuda.h>

#include "mla_common.cuh"
#include "mla_tiles.cuh"
#include "mla_mma.cuh"

namespace mla {

namespace mmak {

constexpr int kGroups = 2;
constexpr int kGroupWarps = 4;
constexpr int kThreads = kGroups * kGroupWarps * 32;  // 256
constexpr int kHalf = kPage / 2;                      // tokens per half page
constexpr int kNSlot = 2;                             // half-page ring per group
constexpr int kChunkBytes = kHalf * 128;              // [32 tokens][64 columns] bf16
constexpr int kTileBytes = 9 * kChunkBytes;           // 36,864
constexpr int kSRow = 20;                             // 16-byte cells per row of a partial-score block: 16
                                                      // column pairs + 4 of padding (a quarter-warp's 16-byte
                                                      // accesses fall in distinct banks)
                                                      // (64-bit accesses by a half-warp hit 32 banks)
constexpr int kSPartBytes = kGroupWarps * 8 * kSRow * 16;  // 10,240: [warp][g][column pair] float4 cells
                                                           // {head g: cols 2c, 2c+1; head g+8: cols 2c, 2c+1}
constexpr int kPBytes = kHeads * 64;                  // [16 heads][32 tokens] bf16, 64-byte rows, swizzled
constexpr int kPrePlan = 64;                          // batches up to this plan before the K1 wait (larger
                                                      // batches fill the SMs with K1, so K2 becomes resident
                                                      // only as K1 ends, and the early scan would delay it)
constexpr int kPreSlots = 1;                          // half pages a group requests before the K1 wait

struct GroupSmem {
    uint64_t full[kNSlot], empty[kNSlot];
    int abort;
    float tmax[kGroupWarps][16];
    float lsum[kGroupWarps][16];
};

constexpr int kOffTile = 0;                                      // [group][slot]
constexpr int kOffS = kOffTile + kGroups * kNSlot * kTileBytes;  // [group]
constexpr int kOffP = kOffS + kGroups * kSPartBytes;             // [group][2]
constexpr int kOffMisc = kOffP + kGroups * 2 * kPBytes;          // [group]
// Pair merge: group 1's first partial, left for group 0 ([4 w][16 n][32 lanes] float4 of O,
// then (m, L) of the 16 heads, then the mbarrier that group 1 arrives on).
constexpr int kOffStash = (kOffMisc + kGroups * (int)sizeof(GroupSmem) + 15) & ~15;
constexpr int kStashOBytes = kGroupWarps * 16 * 32 * 16;         // 32,768
constexpr int kStashBytes = kStashOBytes + kHeads * 8 + 16;
constexpr int kSmemBytes = kOffStash + kStashBytes + 1024;
// kPLo: the low halves of P, [group][2] blocks laid out as the P blocks
constexpr int kOffPLo = (kOffStash + kStashBytes + 127) & ~127;
constexpr int kSmemBytesPLo = kOffPLo + kGroups * 2 * kPBytes + 1024;
static_assert(kSmemBytesPLo <= 232448, "K2 (mma) shared memory exceeds 227 KB");
constexpr int smem_bytes(bool plo) { return plo ? kSmemBytesPLo : kSmemBytes; }
static_assert(kTileBytes % 1024 == 0 && kOffS % 1024 == 0, "TMA slots must stay 1024-byte aligned");

// Zero the bf16 halves of a B fragment register whose token index is >= valid.
__device__ __forceinline__ uint32_t mask_pair(uint32_t v, int tok_lo, int valid) {
    if (tok_lo >= valid) return 0u;
    if (tok_lo + 1 >= valid) return v & 0x0000FFFFu;
    return v;
}

// Byte offset of (head, 16-byte unit u < 4) in a P block: 64-byte rows whose units
// are XOR-swizzled with bits 1-2 of the head, so that the 8 rows an ldmatrix
// reads, and the 8 rows a warp's stores touch, fall in distinct banks.
__device__ __forceinline__ int p_offset(int head, int u) { return head * 64 + ((u ^ ((head >> 1) & 3)) << 4); }

}  // namespace mmak

template <bool kQLo, bool kPLo>
__global__ void __launch_bounds__(mmak::kThreads, 1)
    k2_attention_mma(const MlaDecodeParams p, const __grid_constant__ CUtensorMap tmap_kv, float scale_log2,
                     int pairs) {
    using namespace mmak;
    MLA_TL_SCOPE(1);
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int grp = warp / kGroupWarps, w = warp % kGroupWarps;
    const int bar_id = 1 + grp;  // named barrier of this group (0 is __syncthreads)
    GroupSmem& S = *reinterpret_cast<GroupSmem*>(smem + kOffMisc + grp * (int)sizeof(GroupSmem));
    uint8_t* tile_s = smem + kOffTile + grp * kNSlot * kTileBytes;
    float* spart = reinterpret_cast<float*>(smem + kOffS + grp * kSPartBytes);
    uint8_t* p_s = smem + kOffP + grp * 2 * kPBytes;
    uint8_t* plo_s = smem + kOffPLo + grp * 2 * kPBytes;  // kPLo only

    const WsLayout ws = ws_layout(p);
    char* wsb = reinterpret_cast<char*>(p.workspace);
    const int32_t* cum = reinterpret_cast<const int32_t*>(wsb + ws.tiles_cum);
    const __nv_bfloat16* qa = reinterpret_cast<const __nv_bfloat16*>(wsb + ws.qa);
    const __nv_bfloat16* qa_lo = reinterpret_cast<const __nv_bfloat16*>(wsb + ws.qa_lo);  // kQLo only
    float* part_ml = reinterpret_cast<float*>(wsb + ws.part_ml);
    float* part_acc = reinterpret_cast<float*>(wsb + ws.part_acc);

    pdl_trigger();
    int vc = blockIdx.x + gridDim.x * grp;  // this group's CTA of the plan (group 1 only if the plan has
                                            // more CTAs than the grid; adjacent to group 0's when paired)
    bool paired = false;                    // adjacent plan CTAs, merged across their boundary (k2_pairs)
    float4* stash_o = reinterpret_cast<float4*>(smem + kOffStash);
    float2* stash_ml = reinterpret_cast<float2*>(smem + kOffStash + kStashOBytes);
    uint64_t* stash_bar = reinterpret_cast<uint64_t*>(smem + kOffStash + kStashOBytes + kHeads * 8);
    if (threadIdx.x == 0) {
        mbar_init(stash_bar, 1);
        fence_mbar_init();
    }
    __syncthreads();
    const bool leader = w == 0 && lane == 0;

    // The leader's look-ahead over half pages (loads run two half pages ahead).
    TileCursor la{};
    uint32_t issued = 0;
    auto issue_next = [&]() {
        const int h = la.index();  // half page h of the request: page h / 2, rows 32 (h % 2) ..
        int page = p.block_table[(int64_t)la.b * p.max_blocks + (h >> 1)];
        if (page < 0 || page >= p.n_pages) { record_error(err_sink(p), MLA_DEV_BAD_PAGE); page = 0; }
        const uint32_t slot = issued % kNSlot;
        mbar_arrive_expect_tx(&S.full[slot], kTileBytes);
        tma_load_4d(tile_s + slot * kTileBytes, &tmap_kv, &S.full[slot], 0, kHalf * (h & 1), 0, page,
                    kCacheEvictFirst);
        ++issued;
        la.next();
    };
    // Would the half page the leader loads next hold the row K1 appends in this step?
    auto holds_new_row = [&]() -> bool {
        if (!new_row_count(p)) return false;
        const int row0 = kHalf * la.index(), nr = p.seq_lens[la.b];
        return nr >= row0 && nr < row0 + kHalf;
    };
    auto init_group = [&]() {
        for (int i = 0; i < kNSlot; ++i) { mbar_init(&S.full[i], 1); mbar_init(&S.empty[i], kGroupWarps); }
        S.abort = 0;
        fence_mbar_init();
        prefetch_tmap(&tmap_kv);
    };

    // Batches of at most kPrePlan requests: the split plan from the step's inputs
    // (row counts, positions, limits; complete before K1 started) before the wait
    // on K1. It equals K1's plan (the same rule, plan_tiles), and the leader already
    // requests its first half pages, except one that holds the row K1 appends, so
    // that those copies overlap K1. Larger batches read K1's plan after the wait.
    __shared__ int32_t pre_cum[kPrePlan + 1];
    __shared__ int32_t pre_tot[kThreads / 32];
    const bool pre = p.batch <= kPrePlan;
    PlanEntry pe{};
    int G = 0;
    const int32_t* cumv = cum;  // the prefix sums the cursors walk
    if (pre) {
        const int b = threadIdx.x;
        const int n = b < p.batch ? plan_tiles(p, b) : 0;
        int incl = n;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int t = __shfl_up_sync(0xffffffffu, incl, o);
            if (lane >= o) incl += t;
        }
        if (lane == 31) pre_tot[warp] = incl;
        __syncthreads();
        int before = 0;
        for (int v = 0; v < warp; ++v) before += pre_tot[v];
        if (b < p.batch) pre_cum[b] = before + incl - n;
        if (threadIdx.x == kThreads - 1) pre_cum[p.batch] = before + incl;
        __syncthreads();
        cumv = pre_cum;
        const int64_t U = pre_cum[p.batch];
        G = (int)(U < (int64_t)p.num_ctas ? U : (int64_t)p.num_ctas);
        paired = pairs && G == p.num_ctas;
        if (paired) vc = 2 * blockIdx.x + grp;
        if (vc < G) {
            pe.u_begin = plan_begin(vc, U, G);
            pe.u_end = plan_begin(vc + 1, U, G);
            int lo = 0, hi = p.batch;  // largest b with cum[b] <= u_begin (skips empty requests)
            while (hi - lo > 1) {
                const int mid = (lo + hi) >> 1;
                if (pre_cum[mid] <= pe.u_begin) lo = mid; else hi = mid;
            }
            pe.b = lo;
            pe.cb0 = pre_cum[lo];
            pe.cb1 = pre_cum[lo + 1];
            if (leader) {
                init_group();
                la.init_at(cumv, p.seq_lens, p.batch, pe, new_row_count(p));
                while (issued < kPreSlots && la.valid() && !holds_new_row()) issue_next();
            }
        }
    }
    pdl_wait();  // the plan, absorbed queries and new rows come from K1
    MLA_TL_WAITED(1);
    if (!pre) {
        // G, and both candidate entries (plain and paired numbering) in one round trip to the plan
        const PlanEntry* ents = reinterpret_cast<const PlanEntry*>(wsb + ws.plan + sizeof(PlanHeader));
        G = reinterpret_cast<const PlanHeader*>(wsb + ws.plan)->G;
        pe = ents[vc < p.num_ctas ? vc : 0];
        const int vp = 2 * (int)blockIdx.x + grp;
        PlanEntry pp{};
        if (pairs) pp = ents[vp < p.num_ctas ? vp : 0];
        paired = pairs && G == p.num_ctas;
        if (paired) { vc = vp; pe = pp; }
    }

    if (vc < G) {
        if (leader && !pre) init_group();
        named_bar_sync(bar_id, kGroupWarps * 32);  // barriers initialised
        volatile int* abort = &S.abort;

        if (leader) {
            if (!pre) la.init_at(cumv, p.seq_lens, p.batch, pe, new_row_count(p));
            while (issued < kNSlot && la.valid()) issue_next();
            MLA_TL_MARK(1, 4);  // first half pages requested
        }
        __syncwarp();  // the leader's warp reconverges before its first .aligned MMA

        TileCursor cur;
        cur.init_at(cumv, p.seq_lens, p.batch, pe, new_row_count(p));
        const int g = lane >> 2, t4 = lane & 3;
        const int m8 = lane >> 3, r8 = lane & 7;  // ldmatrix: matrix index, row in matrix
        const uint32_t tile_addr = smem_u32(tile_s), p_addr = smem_u32(p_s), plo_addr = smem_u32(plo_s);

        uint32_t qf[9][4];                     // Q fragments, k-steps [9w, 9w+9)
        uint32_t ql[kQLo ? 9 : 1][4];          // kQLo: fragments of the low half of q_c (latent k-steps only)
        float o[16][4];                        // O_w: 16 latent tiles of 8
        float m_run[2], l_run[2];              // heads g, g+8
        int rows_b = 0;                        // rows attended by the current request
        uint32_t i = 0;                        // half pages consumed
        bool ok = true;
        float seg_L[2] = {0.f, 0.f};           // row sums of the last segment, heads g, g+8
        // The partial (m, L, unnormalised O) of this group's segment into slot s.
        auto write_partial = [&](int64_t s) {
            if (w == 0 && t4 == 0) {
                part_ml[(s * kHeads + g) * 2 + 0] = m_run[0];
                part_ml[(s * kHeads + g) * 2 + 1] = seg_L[0];
                part_ml[(s * kHeads + g + 8) * 2 + 0] = m_run[1];
                part_ml[(s * kHeads + g + 8) * 2 + 1] = seg_L[1];
            }
            float* acc = part_acc + s * kHeads * kLora + 128 * w + 2 * t4;
#pragma unroll
            for (int n = 0; n < 16; ++n) {
                *reinterpret_cast<float2*>(acc + g * kLora + 8 * n) = make_float2(o[n][0], o[n][1]);
                *reinterpret_cast<float2*>(acc + (g + 8) * kLora + 8 * n) = make_float2(o[n][2], o[n][3]);
            }
        };
        // Row count and Q fragments of request b (the first half page of each segment needs them).
        auto load_query = [&](int b) {
            rows_b = p.seq_lens[b] + new_row_count(p);
            const __nv_bfloat16* qrow = qa + (int64_t)b * kQRows * kRow + 144 * w + 2 * t4;
#pragma unroll
            for (int j = 0; j < 9; ++j) {
                const __nv_bfloat16* q0 = qrow + 16 * j;
                qf[j][0] = *reinterpret_cast<const uint32_t*>(q0 + g * kRow);
                qf[j][1] = *reinterpret_cast<const uint32_t*>(q0 + (g + 8) * kRow);
                qf[j][2] = *reinterpret_cast<const uint32_t*>(q0 + g * kRow + 8);
                qf[j][3] = *reinterpret_cast<const uint32_t*>(q0 + (g + 8) * kRow + 8);
            }
            if constexpr (kQLo) {
                const __nv_bfloat16* lrow = qa_lo + (int64_t)b * kQRows * kLora + 144 * w + 2 * t4;
#pragma unroll
                for (int j = 0; j < 9; ++j) {
                    if (144 * w + 16 * j < kLora) {
                        const __nv_bfloat16* l0 = lrow + 16 * j;
                        ql[j][0] = *reinterpret_cast<const uint32_t*>(l0 + g * kLora);
                        ql[j][1] = *reinterpret_cast<const uint32_t*>(l0 + (g + 8) * kLora);
                        ql[j][2] = *reinterpret_cast<const uint32_t*>(l0 + g * kLora + 8);
                        ql[j][3] = *reinterpret_cast<const uint32_t*>(l0 + (g + 8) * kLora + 8);
                    } else {
                        ql[j][0] = ql[j][1] = ql[j][2] = ql[j][3] = 0u;
                    }
                }
            }
        };
        bool q_next = false;  // this segment's query was requested in the previous segment's epilogue
        for (; ok && cur.valid(); cur.next()) {
            const bool first = cur.first(), last = cur.last();
            if (first && !q_next) load_query(cur.b);
            q_next = false;
            const int hvalid = min(kHalf, rows_b - kHalf * cur.index());  // valid tokens of this half page
            if (first) {
#pragma unroll
                for (int n = 0; n < 16; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;
                m_run[0] = m_run[1] = -INFINITY;
                l_run[0] = l_run[1] = 0.f;
            }
            {
                const bool tile_first = first;
                const uint32_t slot = i % kNSlot;
                if (!mbar_wait(&S.full[slot], (i / kNSlot) & 1, abort, err_sink(p))) { ok = false; break; }
                if (i == 0 && w == 0) MLA_TL_MARK(1, 5);  // first half page landed
                const uint32_t tbase = tile_addr + slot * kTileBytes;

                // ---- partial scores over this warp's 144 columns, the 32 tokens ----
                float sacc[4][4];
#pragma unroll
                for (int n = 0; n < 4; ++n) sacc[n][0] = sacc[n][1] = sacc[n][2] = sacc[n][3] = 0.f;
#pragma unroll
                for (int j = 0; j < 9; ++j) {
                    const int k = 144 * w + 16 * j;
                    const int chunk = k >> 6, unit = ((k & 63) >> 3) + (m8 & 1);
#pragma unroll
                    for (int q = 0; q < 2; ++q) {  // token tiles 2q, 2q+1
                        const int tok = 16 * q + (m8 >> 1) * 8 + r8;
                        uint32_t b00, b01, b10, b11;
                        ldsm_x4(tbase + chunk * kChunkBytes + tok * 128 + ((unit ^ r8) << 4), b00, b01, b10, b11);
                        mma16816(sacc[2 * q], qf[j], b00, b01);
                        mma16816(sacc[2 * q + 1], qf[j], b10, b11);
                        if constexpr (kQLo) {
                            if (k < kLora) {  // warp-uniform: the q_pe columns have no low half
                                mma16816(sacc[2 * q], ql[kQLo ? j : 0], b00, b01);
                                mma16816(sacc[2 * q + 1], ql[kQLo ? j : 0], b10, b11);
                            }
                        }
                    }
                }
                // ---- exchange: every warp publishes its partials, then sums its 8 tokens ----
                {
                    float4* mine = reinterpret_cast<float4*>(spart) + w * (8 * kSRow) + g * kSRow;
#pragma unroll
                    for (int n = 0; n < 4; ++n)  // column pair 4n + t4: cols 8n + 2t4, +1
                        mine[4 * n + t4] = make_float4(sacc[n][0], sacc[n][1], sacc[n][2], sacc[n][3]);
                }
                named_bar_sync(bar_id, kGroupWarps * 32);
                float s[4];  // tokens 8w + 2t4 + {0,1}: [0..1] head g, [2..3] head g+8
                {
                    const int col = 8 * w + 2 * t4;
                    float2 lo = make_float2(0.f, 0.f), hi = make_float2(0.f, 0.f);
#pragma unroll
                    for (int v = 0; v < kGroupWarps; ++v) {
                        const float4 x = reinterpret_cast<const float4*>(spart)[(v * 8 + g) * kSRow + 4 * w + t4];
                        lo.x += x.x; lo.y += x.y; hi.x += x.z; hi.y += x.w;
                    }
                    s[0] = col < hvalid ? lo.x * scale_log2 : -INFINITY;
                    s[1] = col + 1 < hvalid ? lo.y * scale_log2 : -INFINITY;
                    s[2] = col < hvalid ? hi.x * scale_log2 : -INFINITY;
                    s[3] = col + 1 < hvalid ? hi.y * scale_log2 : -INFINITY;
                }
                // ---- probabilities (bf16) for this warp's 8 tokens -> P buffer ----
                uint8_t* pb = p_s + (i & 1) * kPBytes;
                float lsum0 = 0.f, lsum1 = 0.f;  // this thread's row-sum terms, heads g, g+8
                auto write_p = [&]() {
                    if constexpr (kPLo) {
                        const float e0 = fast_exp2(s[0] - m_run[0]), e1 = fast_exp2(s[1] - m_run[0]);
                        const float e2 = fast_exp2(s[2] - m_run[1]), e3 = fast_exp2(s[3] - m_run[1]);
                        const float h0 = bf16_round(e0), h1 = bf16_round(e1), h2 = bf16_round(e2),
                                    h3 = bf16_round(e3);
                        lsum0 = e0 + e1;
                        lsum1 = e2 + e3;
                        uint8_t* pl = plo_s + (i & 1) * kPBytes;
                        *reinterpret_cast<uint32_t*>(pb + p_offset(g, w) + 4 * t4) = pack_bf16(h0, h1);
                        *reinterpret_cast<uint32_t*>(pb + p_offset(g + 8, w) + 4 * t4) = pack_bf16(h2, h3);
                        *reinterpret_cast<uint32_t*>(pl + p_offset(g, w) + 4 * t4) = pack_bf16(e0 - h0, e1 - h1);
                        *reinterpret_cast<uint32_t*>(pl + p_offset(g + 8, w) + 4 * t4) = pack_bf16(e2 - h2, e3 - h3);
                    } else {
                        const float e0 = bf16_round(fast_exp2(s[0] - m_run[0]));
                        const float e1 = bf16_round(fast_exp2(s[1] - m_run[0]));
                        const float e2 = bf16_round(fast_exp2(s[2] - m_run[1]));
                        const float e3 = bf16_round(fast_exp2(s[3] - m_run[1]));
                        lsum0 = e0 + e1;
                        lsum1 = e2 + e3;
                        *reinterpret_cast<uint32_t*>(pb + p_offset(g, w) + 4 * t4) = pack_bf16(e0, e1);
                        *reinterpret_cast<uint32_t*>(pb + p_offset(g + 8, w) + 4 * t4) = pack_bf16(e2, e3);
                    }
                };
                // ---- running max (log2 domain), lazy rescale ----
                // Past a segment's first half page the probabilities are written with the running
                // max first; one barrier with an OR-reduction then both publishes them and says
                // whether any score exceeded the max by more than 2^8. Only then (rare) the group
                // exchanges the tile maxima, rescales, and writes them again behind one more barrier.
                bool exchange = tile_first;
                if (!tile_first) {
                    const bool ex = fmaxf(s[0], s[1]) > m_run[0] + 8.f || fmaxf(s[2], s[3]) > m_run[1] + 8.f;
                    write_p();
                    exchange = bar_red_or(bar_id, kGroupWarps * 32, ex);
                }
                if (exchange) {
                    float mx0 = fmaxf(s[0], s[1]), mx1 = fmaxf(s[2], s[3]);
                    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
                    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
                    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
                    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
                    if (t4 == 0) { S.tmax[w][g] = mx0; S.tmax[w][g + 8] = mx1; }
                    named_bar_sync(bar_id, kGroupWarps * 32);
                    const float t0 = fmaxf(fmaxf(S.tmax[0][g], S.tmax[1][g]), fmaxf(S.tmax[2][g], S.tmax[3][g]));
                    const float t1 =
                        fmaxf(fmaxf(S.tmax[0][g + 8], S.tmax[1][g + 8]), fmaxf(S.tmax[2][g + 8], S.tmax[3][g + 8]));
                    const float n0 = fmaxf(m_run[0], t0), n1 = fmaxf(m_run[1], t1);
                    if (!tile_first) {
                        const float f0 = fast_exp2(m_run[0] - n0), f1 = fast_exp2(m_run[1] - n1);
#pragma unroll
                        for (int n = 0; n < 16; ++n) { o[n][0] *= f0; o[n][1] *= f0; o[n][2] *= f1; o[n][3] *= f1; }
                        l_run[0] *= f0;
                        l_run[1] *= f1;
                    }
                    m_run[0] = n0;
                    m_run[1] = n1;
                    write_p();
                    named_bar_sync(bar_id, kGroupWarps * 32);
                }
                l_run[0] += lsum0;
                l_run[1] += lsum1;

                // ---- O_w += P C[:, 128w : 128w+128] ----
                const uint32_t pbase = p_addr + (i & 1) * kPBytes;
#pragma unroll
                for (int ks = 0; ks < 2; ++ks) {
                    uint32_t a[4], al[4];
                    ldsm_x4(pbase + p_offset((m8 & 1) * 8 + r8, 2 * ks + (m8 >> 1)), a[0], a[1], a[2], a[3]);
                    if constexpr (kPLo)
                        ldsm_x4(plo_addr + (i & 1) * kPBytes + p_offset((m8 & 1) * 8 + r8, 2 * ks + (m8 >> 1)), al[0],
                                al[1], al[2], al[3]);
                    const int tok = 16 * ks + (m8 & 1) * 8 + r8;
#pragma unroll
                    for (int pp = 0; pp < 8; ++pp) {  // latent tiles 2pp, 2pp+1 of this warp
                        const int chunk = 2 * w + (pp >> 2);
                        const int unit = 2 * (pp & 3) + (m8 >> 1);
                        uint32_t b00, b01, b10, b11;
                        ldsm_x4_t(tbase + chunk * kChunkBytes + tok * 128 + ((unit ^ r8) << 4), b00, b01, b10, b11);
                        if (hvalid < kHalf) {
                            const int tl = 16 * ks + 2 * t4;
                            b00 = mask_pair(b00, tl, hvalid);
                            b10 = mask_pair(b10, tl, hvalid);
                            b01 = mask_pair(b01, tl + 8, hvalid);
                            b11 = mask_pair(b11, tl + 8, hvalid);
                        }
                        mma16816(o[2 * pp], a, b00, b01);
                        mma16816(o[2 * pp + 1], a, b10, b11);
                        if constexpr (kPLo) {
                            mma16816(o[2 * pp], al, b00, b01);
                            mma16816(o[2 * pp + 1], al, b10, b11);
                        }
                    }
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(&S.empty[slot]);
                // the leader refills this slot with the half page two ahead once all four warps released it
                bool refill_ok = true;
                if (leader && la.valid()) {
                    refill_ok = mbar_wait(&S.empty[slot], (i / kNSlot) & 1, abort, err_sink(p));
                    if (refill_ok) issue_next();
                }
                if (!__shfl_sync(0xffffffffu, refill_ok, 0)) { ok = false; break; }  // reconverges the warp
                ++i;
            }

            if (last) {
                // The next segment's row count and query, requested now (the fragments are dead
                // after this half page's score MMAs) so that their latency overlaps this epilogue.
                if (cur.u + 1 < cur.u_end) {
                    TileCursor nx = cur;
                    nx.next();
                    load_query(nx.b);
                    q_next = true;
                }
                // ---- partial of (request, this virtual CTA): m, l, unnormalised O ----
                float l0 = l_run[0], l1 = l_run[1];
                l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
                l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
                l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
                l1 += __shfl_xor_sync(0xffffffffu, l1, 2);
                if (t4 == 0) { S.lsum[w][g] = l0; S.lsum[w][g + 8] = l1; }
                named_bar_sync(bar_id, kGroupWarps * 32);
                seg_L[0] = (S.lsum[0][g] + S.lsum[1][g]) + (S.lsum[2][g] + S.lsum[3][g]);
                seg_L[1] = (S.lsum[0][g + 8] + S.lsum[1][g + 8]) + (S.lsum[2][g + 8] + S.lsum[3][g + 8]);
                // Pair merge: the boundary between plan CTAs 2k and 2k + 1 falls inside a request
                // when group 1's first segment started before its range and group 0's last
                // segment goes on past its range. Group 1 leaves that partial in shared memory;
                // group 0 merges it into its own (rescaled to the larger max) and writes slot 2k + b.
                if (paired && grp == 1 && cur.seg == 0 && cur.u_begin > cur.cb0) {
#pragma unroll
                    for (int n = 0; n < 16; ++n)
                        stash_o[(w * 16 + n) * 32 + lane] = make_float4(o[n][0], o[n][1], o[n][2], o[n][3]);
                    if (w == 0 && t4 == 0) {
                        stash_ml[g] = make_float2(m_run[0], seg_L[0]);
                        stash_ml[g + 8] = make_float2(m_run[1], seg_L[1]);
                    }
                    named_bar_sync(bar_id, kGroupWarps * 32);
                    if (leader) mbar_arrive(stash_bar);
                } else {
                    if (paired && grp == 0 && cur.u == cur.u_end - 1 && cur.u_end < cur.cb1 &&
                        mbar_wait(stash_bar, 0, abort, err_sink(p))) {
                        const float2 p0 = stash_ml[g], p1 = stash_ml[g + 8];
                        const float n0 = fmaxf(m_run[0], p0.x), n1 = fmaxf(m_run[1], p1.x);
                        const float a0 = exp2f(m_run[0] - n0), b0 = exp2f(p0.x - n0);
                        const float a1 = exp2f(m_run[1] - n1), b1 = exp2f(p1.x - n1);
#pragma unroll
                        for (int n = 0; n < 16; ++n) {
                            const float4 x = stash_o[(w * 16 + n) * 32 + lane];
                            o[n][0] = o[n][0] * a0 + x.x * b0;
                            o[n][1] = o[n][1] * a0 + x.y * b0;
                            o[n][2] = o[n][2] * a1 + x.z * b1;
                            o[n][3] = o[n][3] * a1 + x.w * b1;
                        }
                        seg_L[0] = seg_L[0] * a0 + p0.y * b0;
                        seg_L[1] = seg_L[1] * a1 + p1.y * b1;
                        m_run[0] = n0;
                        m_run[1] = n1;
                    }
                    write_partial((int64_t)vc + cur.b);
                }
                // the lsum buffer is reused by the next segment's epilogue only after
                // at least one more half page's barriers, which every warp passes after this read
            }
        }
        // Drain: every copy the leader issued must land before the CTA's shared memory is released.
        if (leader) {
            for (uint32_t sl = 0; sl < kNSlot; ++sl) {
                const uint32_t fills = issued / kNSlot + (sl < issued % kNSlot ? 1u : 0u);
                if (fills) mbar_drain(&S.full[sl], (fills - 1) & 1, err_sink(p));
            }
        }
    }
    __syncthreads();
}

int k2_mma_smem_bytes() { return mmak::kSmemBytes; }

cudaError_t k2_mma_configure() {
    cudaError_t e = cudaFuncSetAttribute(k2_attention_mma<false, false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         mmak::smem_bytes(false));
    if (e == cudaSuccess)
        e = cudaFuncSetAttribute(k2_attention_mma<true, false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 mmak::smem_bytes(false));
    if (e == cudaSuccess)
        e = cudaFuncSetAttribute(k2_attention_mma<false, true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 mmak::smem_bytes(true));
    if (e == cudaSuccess)
        e = cudaFuncSetAttribute(k2_attention_mma<true, true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 mmak::smem_bytes(true));
    return e;
}

cudaError_t launch_attention_mma(const MlaDecodeParams& p, const CUtensorMap& tmap_kv, float scale_log2,
                                 int sm_count, cudaStream_t stream) {
    static_assert(mmak::kGroups == 2, "k2_grid assumes two plan CTAs per CTA");
    const int grid = k2_grid(p.num_ctas, sm_count);
    const bool qlo = (p.flags & MLA_FLAG_QC_HILO) != 0, plo = (p.flags & MLA_FLAG_P_HILO) != 0;
    auto kern = qlo ? (plo ? k2_attention_mma<true, true> : k2_attention_mma<true, false>)
                    : (plo ? k2_attention_mma<false, true> : k2_attention_mma<false, false>);
    const cudaError_t e = launch_pdl(kern, dim3(grid), dim3(mmak::kThreads), mmak::smem_bytes(plo), stream, p,
                                     tmap_kv, scale_log2, k2_pairs(p, sm_count) ? 1 : 0);
    if (e != cudaSuccess) return e;
    return cudaGetLastError();
}

}  // namespace mla
