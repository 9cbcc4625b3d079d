// K1 — the attention task's prologue, once per request (not once per head x
// chunk as in the reference, which re-derives it in every attention task).
//
//  * kv_post: RMSNorm of c_new with HF's two bf16 roundings, RoPE of k_pe_new,
//    bf16 row appended to the request's page (reference_decode.py:231-237,
//    src/kernels/attention.h:62-90);
//  * q_pe RoPE, bf16-rounded (reference_decode.py:235);
//  * q-absorb q_c[h] = q_nope[h] @ W_UK[h] with fp32 accumulation
//    (reference_decode.py:250, attention.h:171-216): per (block of 64 requests,
//    head, quarter of the latent) an m16n8k16 GEMM [64 requests x 128] x
//    [128 x 128] against a 32 KB slice of W_UK[h] staged by one TMA box; q_nope
//    and W_UK are bf16 already, so the products are exact; q_c is stored bf16 as
//    an operand of the attention kernel's score contraction (with
//    MLA_FLAG_QC_HILO also its remainder, as a second bf16 operand);
//  * the split plan: prefix sum of tiles per request (plan_unit_rows: 32-row half
//    pages for the default split-KV kernel, 64-row pages for the others), consumed by K2/K3.
//
// One 1-D grid with two kinds of CTA:
//   [0, n_absorb)  absorb: (request block of 64, head, quarter of the latent
//                  columns). Warps 0-3 stage q_nope and run the MMAs against a
//                  32 KB W_UK slice; warp 4 does the per-request work of one
//                  request of the block (q_pe RoPE, kv_post, cache append).
//   last           planner
#include <cuda.h>

#include "mla_common.cuh"
#include "mla_mma.cuh"
#include "mla_rowops.cuh"

namespace mla {

constexpr int kReqBlock = 64;                         // requests per absorb CTA (4 m16 tiles)
constexpr int kQuarters = kLora / kK1LatQ;            // 4
constexpr int kK1MmaWarps = 4;
constexpr int kK1Threads = (kK1MmaWarps + 1) * 32;    // + the per-request warp
constexpr int kWukBytes = kNope * kK1LatQ * 2;        // 32768: [2 column blocks][128 d][128 B], swizzled
constexpr int kQnBytes = kReqBlock * kNope * 2;       // 16384: [64 requests][128] bf16, 256-byte rows, swizzled
constexpr int kK1SmemBytes = kWukBytes + kQnBytes + 64 + 1024;
static_assert(kReqBlock == kHeads * kQuarters, "each absorb CTA of a block owns one request's row work");

struct K1Grid {
    int n_rb, n_absorb, total;
    __host__ __device__ explicit K1Grid(int batch) {
        n_rb = (batch + kReqBlock - 1) / kReqBlock;
        n_absorb = n_rb * kHeads * kQuarters;
        total = n_absorb + 1;
    }
};

// Prefix sum of tiles per request (one CTA). Invalid positions are recorded
// and given zero tiles, so no later kernel reads outside the block table.
// cum_s (kCumSmem entries of shared memory) receives a copy when batch + 1 fits.
constexpr int kCumSmem = (kK1SmemBytes - 1024) / 4;  // what is left after aligning the base to 1024 bytes
__device__ void plan_scan(const MlaDecodeParams& p, int32_t* cum, int32_t* cum_s) {
    __shared__ int32_t warp_tot[kK1Threads / 32];
    __shared__ int32_t carry;
    const bool stage = p.batch + 1 <= kCumSmem;
    if (threadIdx.x == 0) carry = 0;
    __syncthreads();
    for (int base = 0; base < p.batch; base += kK1Threads) {
        const int b = base + threadIdx.x;
        int n = 0;
        if (b < p.batch) {
            if (!request_ok(p, b)) record_error(err_sink(p), MLA_DEV_BAD_POSITION);
            else n = plan_tiles(p, b);
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
        if (b < p.batch) {
            cum[b] = before + incl - n;
            if (stage) cum_s[b] = before + incl - n;
        }
        __syncthreads();
        if (threadIdx.x == kK1Threads - 1) carry = before + incl;
        __syncthreads();
    }
    if (threadIdx.x == 0) {
        cum[p.batch] = carry;
        if (stage) cum_s[p.batch] = carry;
    }
}

// Per plan CTA of the split-KV kernel: its tile range and first request (the same
// search TileCursor::init does, here once per CTA instead of in every thread of
// the split-KV kernel after its grid-dependency wait).
__device__ void plan_entries(const MlaDecodeParams& p, const int32_t* cum, const int32_t* cum_s, char* plan) {
    __syncthreads();  // cum / cum_s complete
    const bool staged = p.batch + 1 <= kCumSmem;
    const int32_t* c = staged ? cum_s : cum;
    const int64_t U = c[p.batch];
    const int G = (int)(U < (int64_t)p.num_ctas ? U : (int64_t)p.num_ctas);
    if (threadIdx.x == 0) {
        PlanHeader* hdr = reinterpret_cast<PlanHeader*>(plan);
        hdr->U = U;
        hdr->G = G;
        hdr->pad = 0;
    }
    PlanEntry* ent = reinterpret_cast<PlanEntry*>(plan + sizeof(PlanHeader));
    for (int vc = threadIdx.x; vc < G; vc += blockDim.x) {
        PlanEntry e;
        e.u_begin = plan_begin(vc, U, G);
        e.u_end = plan_begin(vc + 1, U, G);
        int lo = 0, hi = p.batch;  // largest b with cum[b] <= u_begin (skips empty requests)
        while (hi - lo > 1) {
            const int mid = (lo + hi) >> 1;
            if (c[mid] <= e.u_begin) lo = mid; else hi = mid;
        }
        e.b = lo;
        e.cb0 = c[lo];
        e.cb1 = c[lo + 1];
        e.pad = 0;
        ent[vc] = e;
    }
}

// The per-request warp's inputs that no earlier kernel writes: the row count and RoPE
// position, the RoPE table rows of that position, the block-table entry of the new
// row and kv_a_layernorm's weight. They are loaded before the wait on the previous
// kernel (positions, tables and weights are the step's inputs, as for the split
// plan that K2 derives before its own wait), so that after the wait only q_pe and
// the raw kv_a row, the previous kernel's output, remain to be loaded.
struct RowPre {
    int pos, rp, page;
    bool ok, append;
    float c0, c1, s0, s1;
    __align__(16) __nv_bfloat16 gw[16];
};

__device__ void request_rows_pre(const MlaDecodeParams& p, int b, int lane, RowPre& r) {
    r.pos = p.seq_lens[b];
    r.rp = p.rope_pos ? p.rope_pos[b] : r.pos;
    r.append = new_row_count(p) != 0;
    const __nv_bfloat16* gam = reinterpret_cast<const __nv_bfloat16*>(p.kv_a_norm_w);
    if (r.append) {
        if ((reinterpret_cast<uintptr_t>(gam) & 15) == 0) {
            reinterpret_cast<uint4*>(r.gw)[0] = reinterpret_cast<const uint4*>(gam)[2 * lane];
            reinterpret_cast<uint4*>(r.gw)[1] = reinterpret_cast<const uint4*>(gam)[2 * lane + 1];
        } else {
#pragma unroll
            for (int k = 0; k < 16; ++k) r.gw[k] = gam[16 * lane + k];
        }
    }
    // request_ok on the loaded values (an invalid request is recorded by the planner)
    r.ok = r.pos >= 0 && r.rp >= 0 && r.rp < p.max_pos && r.pos + new_row_count(p) <= p.max_blocks * kPage;
    r.page = 0;
    if (!r.ok) return;
    const float* cs = p.rope_cos + (int64_t)r.rp * kRope;
    const float* sn = p.rope_sin + (int64_t)r.rp * kRope;
    r.c0 = cs[lane]; r.c1 = cs[32 + lane]; r.s0 = sn[lane]; r.s1 = sn[32 + lane];
    if (r.append) r.page = p.block_table[(int64_t)b * p.max_blocks + r.pos / kPage];
}

// One warp, after the wait: q_pe RoPE of request b, then (unless the call stores no
// row) kv_post + the cache append at local row seq_lens[b].
__device__ void request_rows(const MlaDecodeParams& p, __nv_bfloat16* qa, int b, int lane, const RowPre& r) {
    if (!r.ok) return;
    const __nv_bfloat16* q = reinterpret_cast<const __nv_bfloat16*>(p.q) + (int64_t)b * p.q_stride;
    __nv_bfloat162 xq[kHeads];
#pragma unroll
    for (int h = 0; h < kHeads; ++h) xq[h] = reinterpret_cast<const __nv_bfloat162*>(q + h * kQHead + kNope)[lane];
    KvPostIn kin;
    if (r.append) {
        const __nv_bfloat16* src = reinterpret_cast<const __nv_bfloat16*>(p.kv_a) + (int64_t)b * p.kv_a_stride;
        kv_post_load(src, nullptr, lane, kin);
#pragma unroll
        for (int k = 0; k < 16; ++k) kin.gw[k] = r.gw[k];
    }

    // q_pe of all 16 heads: lane j rotates pair j
    __nv_bfloat16* qrow = qa + (int64_t)b * kQRows * kRow;
#pragma unroll
    for (int h = 0; h < kHeads; ++h) {
        float lo, hi;
        rope_pair_r(__low2float(xq[h]), __high2float(xq[h]), r.c0, r.s0, r.c1, r.s1, lo, hi);
        qrow[h * kRow + kLora + lane] = __float2bfloat16_rn(lo);
        qrow[h * kRow + kLora + 32 + lane] = __float2bfloat16_rn(hi);
    }
    if (!r.append) return;

    __align__(16) __nv_bfloat16 outc[16];
    float lo, hi;
    kv_post_finish_r(kin, p.rms_eps, r.c0, r.s0, r.c1, r.s1, lane, outc, lo, hi);
    if (r.page < 0 || r.page >= p.n_pages) {
        if (lane == 0) record_error(err_sink(p), MLA_DEV_BAD_PAGE);
        return;
    }
    kv_post_store(reinterpret_cast<__nv_bfloat16*>(p.kv_cache) + ((int64_t)r.page * kPage + r.pos % kPage) * kRow,
                  outc, lo, hi, lane);
}

__global__ void __launch_bounds__(kK1Threads) k1_prologue(const MlaDecodeParams p,
                                                            const __grid_constant__ CUtensorMap tmap_wuk) {
    MLA_TL_SCOPE(0);
    const WsLayout ws = ws_layout(p);
    char* wsb = reinterpret_cast<char*>(p.workspace);
    __nv_bfloat16* qa = reinterpret_cast<__nv_bfloat16*>(wsb + ws.qa);
    const K1Grid g(p.batch);
    const int cta = blockIdx.x;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* w_s = smem;
    uint8_t* q_s = smem + kWukBytes;
    uint64_t* bar = reinterpret_cast<uint64_t*>(q_s + kQnBytes);
    const int rb = cta / (kHeads * kQuarters), c_in = cta % (kHeads * kQuarters);
    const int h = c_in / kQuarters, j = c_in % kQuarters;
    if (cta != g.total - 1 && threadIdx.x == 0) {  // W_UK is a weight: no kernel writes it, so before pdl_wait
        mbar_init(bar, 1);
        fence_mbar_init();
        mbar_arrive_expect_tx(bar, kWukBytes);
        tma_load_3d(w_s, &tmap_wuk, bar, 0, h * kKvbHead, kK1WukBlocks * j, kCacheEvictLast);
    }
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int b0 = rb * kReqBlock;
    const int nreq = min(kReqBlock, p.batch - b0);
    if (cta != g.total - 1 && warp == kK1MmaWarps) {  // the per-request work of request b0 + c_in
        RowPre pre;
        if (c_in < nreq) request_rows_pre(p, b0 + c_in, lane, pre);
        pdl_wait();  // q and kv_a come from the previous kernel
        MLA_TL_WAITED(0);
        pdl_trigger();
        if (c_in < nreq) request_rows(p, qa, b0 + c_in, lane, pre);
        MLA_TL_MARK(0, 5);
        return;  // joins no barrier
    }
    pdl_wait();     // q, kv_a and the cache come from earlier work on the stream
    MLA_TL_WAITED(0);
    pdl_trigger();  // K2 may become resident now; it waits for this grid before reading its output

    if (cta == g.total - 1) {
        int32_t* cum = reinterpret_cast<int32_t*>(wsb + ws.tiles_cum);
        int32_t* cum_s = reinterpret_cast<int32_t*>(smem);
        plan_scan(p, cum, cum_s);
        plan_entries(p, cum, cum_s, wsb + ws.plan);
        return;
    }

    // ---- absorb CTA: q_c[b][h][128j + l] = q_nope[b][h] @ W_UK[h][:, 128j + l] ----
    // q_nope [64][128] -> shared, 256-byte rows with 16-byte units XOR (row & 7)
    {
        const __nv_bfloat16* q = reinterpret_cast<const __nv_bfloat16*>(p.q);
        constexpr int kUnits = kReqBlock * (kNope / 8);  // 16-byte units
        constexpr int kPer = kUnits / (kK1MmaWarps * 32);
        const bool vec = (reinterpret_cast<uintptr_t>(q) & 15) == 0 && (p.q_stride & 7) == 0;
        uint4 v[kPer];
#pragma unroll
        for (int k = 0; k < kPer; ++k) {
            const int i = threadIdx.x + k * kK1MmaWarps * 32;
            const int r = i >> 4, u = i & 15;
            const __nv_bfloat16* src = q + (int64_t)(b0 + r) * p.q_stride + h * kQHead + u * 8;
            v[k] = make_uint4(0u, 0u, 0u, 0u);
            if (r < nreq) {
                if (vec) {
                    v[k] = *reinterpret_cast<const uint4*>(src);
                } else {
                    const uint32_t* s32 = reinterpret_cast<const uint32_t*>(src);
                    v[k] = make_uint4(s32[0], s32[1], s32[2], s32[3]);
                }
            }
        }
#pragma unroll
        for (int k = 0; k < kPer; ++k) {
            const int i = threadIdx.x + k * kK1MmaWarps * 32;
            const int r = i >> 4, u = i & 15;
            *reinterpret_cast<uint4*>(q_s + r * 256 + ((u ^ (r & 7)) << 4)) = v[k];
        }
    }
    named_bar_sync(1, kK1MmaWarps * 32);  // q_nope staged, barrier initialised
    {
        int dummy = 0;
        if (!mbar_wait(bar, 0, &dummy, err_sink(p))) return;
    }
    // D[64 requests][128] = A[64][128 d] x W_UK[h][128 d][128 l]; warp w owns l in [32w, 32w+32)
    const int gq = lane >> 2, t4 = lane & 3, m8 = lane >> 3, r8 = lane & 7;
    const int n_mt = (nreq + 15) >> 4;
    const uint32_t wb = smem_u32(w_s), qb = smem_u32(q_s);
    float acc[4][4][4];
#pragma unroll
    for (int mt = 0; mt < 4; ++mt)
#pragma unroll
        for (int n = 0; n < 4; ++n) acc[mt][n][0] = acc[mt][n][1] = acc[mt][n][2] = acc[mt][n][3] = 0.f;
#pragma unroll
    for (int ks = 0; ks < kNope / 16; ++ks) {
        const int d = 16 * ks + (m8 & 1) * 8 + r8;
        uint32_t bw[2][4];
#pragma unroll
        for (int np = 0; np < 2; ++np) {  // latent tiles 2np, 2np+1 of this warp
            const int l = 32 * warp + 16 * np + (m8 >> 1) * 8;
            ldsm_x4_t(wb + (l >> 6) * (kNope * 128) + d * 128 + ((((l & 63) >> 3) ^ r8) << 4), bw[np][0], bw[np][1],
                      bw[np][2], bw[np][3]);
        }
#pragma unroll
        for (int mt = 0; mt < 4; ++mt) {
            if (mt < n_mt) {
                uint32_t a[4];
                const int row = 16 * mt + (m8 & 1) * 8 + r8, col = 16 * ks + (m8 >> 1) * 8;
                ldsm_x4(qb + row * 256 + ((((col >> 3) ^ (row & 7))) << 4), a[0], a[1], a[2], a[3]);
#pragma unroll
                for (int np = 0; np < 2; ++np) {
                    mma16816(acc[mt][2 * np], a, bw[np][0], bw[np][1]);
                    mma16816(acc[mt][2 * np + 1], a, bw[np][2], bw[np][3]);
                }
            }
        }
    }
    // MLA_FLAG_QC_HILO: the remainder q_c - bf16(q_c), rounded to bf16, into qa_lo
    __nv_bfloat16* qa_lo = (p.flags & MLA_FLAG_QC_HILO) ? reinterpret_cast<__nv_bfloat16*>(wsb + ws.qa_lo) : nullptr;
    auto lo2 = [](float x, float y) { return pack_bf16(x - bf16_round(x), y - bf16_round(y)); };
#pragma unroll
    for (int mt = 0; mt < 4; ++mt) {
        if (mt >= n_mt) break;
#pragma unroll
        for (int n = 0; n < 4; ++n) {
            const int l = kK1LatQ * j + 32 * warp + 8 * n + 2 * t4;
            const int r0 = 16 * mt + gq, r1 = r0 + 8;
            if (r0 < nreq) {
                *reinterpret_cast<uint32_t*>(qa + ((int64_t)(b0 + r0) * kQRows + h) * kRow + l) =
                    pack_bf16(acc[mt][n][0], acc[mt][n][1]);
                if (qa_lo)
                    *reinterpret_cast<uint32_t*>(qa_lo + ((int64_t)(b0 + r0) * kQRows + h) * kLora + l) =
                        lo2(acc[mt][n][0], acc[mt][n][1]);
            }
            if (r1 < nreq) {
                *reinterpret_cast<uint32_t*>(qa + ((int64_t)(b0 + r1) * kQRows + h) * kRow + l) =
                    pack_bf16(acc[mt][n][2], acc[mt][n][3]);
                if (qa_lo)
                    *reinterpret_cast<uint32_t*>(qa_lo + ((int64_t)(b0 + r1) * kQRows + h) * kLora + l) =
                        lo2(acc[mt][n][2], acc[mt][n][3]);
            }
        }
    }
    MLA_TL_MARK(0, 4);
}

cudaError_t k1_configure() {
    return cudaFuncSetAttribute(k1_prologue, cudaFuncAttributeMaxDynamicSharedMemorySize, kK1SmemBytes);
}

cudaError_t launch_prologue(const MlaDecodeParams& p, const CUtensorMap& tmap_wuk, cudaStream_t stream) {
    const K1Grid g(p.batch);
    return launch_pdl(k1_prologue, dim3(g.total), dim3(kK1Threads), kK1SmemBytes, stream, p, tmap_wuk);
}

}  // namespace mla
