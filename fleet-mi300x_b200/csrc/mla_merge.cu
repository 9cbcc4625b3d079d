// K3 — merge of the split-KV partials and the W_UV up-projection.
//
// Follows merge_and_uv (src/kernels/attention.h:358-411): global max over the
// partials, rescaled sum in a fixed order, divide by the rescaled sum of
// exps, then o[h] = o_c[h] @ W_UV[h]^T with the bf16 epilogue
// (reference_decode.py:252-256). Partials are merged in CTA order, so the
// result is bitwise reproducible for a fixed split plan.
//
// Grid: x = head (x cluster rank), y = block of requests; 256 threads. A CTA
// stages its rows of W_UV[h] (kv_b rows [256h+128, 256h+256), 512 columns) with
// one TMA box while it merges the partials of its requests into o_c (fp32), then
// runs out[r][v] = sum_l o_c[r][l] W_UV[h][v][l] as m16n8k16 MMAs with the
// requests on M. o_c enters the MMA as a bf16 hi/lo pair (hi = bf16(o_c),
// lo = bf16(o_c - hi)), two MMAs per step, so the product keeps ~16 mantissa
// bits of o_c, as the reference's fp32 GEMV does. Three forms (k3_launch):
//   * cluster form, batches of at most 4 blocks of 16: a thread-block cluster of 4
//     CTAs per (head, block), each folding a quarter of the partials and owning 32
//     rows of W_UV; the folds meet through distributed shared memory. Batches of
//     5-16 run as two blocks of 4 or 8 requests (k3_cluster_rpb);
//   * plain form, one CTA per (head, block of 16), while that grid fits one wave;
//   * plain form in blocks of 32 (two m16 tiles on one staged W_UV[h]) beyond.
// Sequence-sharded steps end here too: shard_out (fp32 partials for a gather) or
// the peer exchange (stores to every rank's buffer; the fused form also combines).
#include <cuda.h>

#include "mla_common.cuh"
#include "mla_mma.cuh"

namespace mla {

namespace k3 {
constexpr int kReq = 16;                          // requests per block (per m16 tile of the W_UV MMA)
constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr int kRedBytes = kWarps * kLora * 4;     // 16384: one fp32 o_c row per warp (warp-group combine)

// kCl CTAs (a thread-block cluster when > 1) share one (head, block of kRq
// requests): each folds every kCl-th partial, and owns kV / kCl rows of W_UV.
// kRq = 32 (plain form only) runs two m16 tiles against one staged W_UV[h].
template <int kCl, int kRq = kReq>
struct Shape {
    static_assert(kRq == kReq || (kRq == 2 * kReq && kCl == 1), "32-request blocks exist in the plain form only");
    static constexpr int kMt = kRq / 16;                       // m16 tiles of requests
    static constexpr int kVRows = kV / kCl;                    // W_UV rows (v) of this CTA
    static constexpr int kWBytes = kVRows * kLora * 2;         // [8 column blocks][kVRows rows][128 B], swizzled
    static constexpr int kABytes = kRq * kLora * 2;            // [kRq requests][512] bf16, 1024-byte rows, swizzled
    static constexpr int kXBytes = kCl > 1 ? kCl * kRq * (kLora + 4) * 4 : 0;  // cluster exchange: per rank
                                                                              // and request acc[512], m, L
    static constexpr int kSmemBytes = kWBytes + 2 * kABytes + kRedBytes + kXBytes + 64 + 1024;
};
constexpr int kClusterCtas = kK3ClusterCtas;  // cluster form: CTAs per (head, request block)
}  // namespace k3

// The cluster form runs when the batch has at most 4 blocks of 16 requests, where
// the plain form would leave most SMs idle.
__host__ __device__ inline bool k3_use_cluster(int batch) { return (batch + k3::kReq - 1) / k3::kReq <= 4; }

// Partial slot s = (c + b) * heads + h: its (m, L) pair and the lane's four
// float4 of acc (latent l = 4 lane + 128 k, k < 4).
__device__ __forceinline__ void load_partial(const float* __restrict__ part_ml, const float* __restrict__ part_acc,
                                             int b, int h, int c, int lane, float2& ml, float4 (&a)[4]) {
    const int64_t s = (int64_t)(c + b) * kHeads + h;
    ml = *reinterpret_cast<const float2*>(part_ml + s * 2);
#pragma unroll
    for (int k = 0; k < 4; ++k) a[k] = reinterpret_cast<const float4*>(part_acc + s * kLora)[lane + 32 * k];
}

// The partials of one request, in fold order: index e < n maps to the plan CTA
// whose slot holds it. Unpaired: c0 + e. Paired (k2_pairs): the split-KV kernel
// merged plan CTA 2k + 1's first partial into 2k's wherever their boundary falls
// inside the request, so the request's partials sit at its first plan CTA c0 and at
// every even plan CTA after it.
struct PartIdx {
    int c0;
    bool paired;
    __device__ __forceinline__ int c(int e) const { return !paired ? c0 + e : (e == 0 ? c0 : 2 * ((c0 >> 1) + e)); }
};

// One step of the online LSE merge: running max m (log2 domain), rescaled sum of
// exps L and unnormalised acc absorb the partial (ml.x = its max, ml.y = its sum).
__device__ __forceinline__ void fold_partial(float2 ml, const float4 (&a)[4], float& m, float& L, float4 (&acc)[4]) {
    const float mn = fmaxf(m, ml.x);
    const float so = exp2f(m - mn), sc = exp2f(ml.x - mn);
    L = L * so + sc * ml.y;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        acc[k].x = acc[k].x * so + sc * a[k].x;
        acc[k].y = acc[k].y * so + sc * a[k].y;
        acc[k].z = acc[k].z * so + sc * a[k].z;
        acc[k].w = acc[k].w * so + sc * a[k].w;
    }
    m = mn;
}

// Fold of the partials c = first, first + stride, ... <= last of (request b,
// head h), in order. Loads are issued kDepth partials (kDepth x 2 KB per warp)
// at a time. (Six or eight at a time measured no faster than four: at one request
// the fold is bound by the bytes each of the 64 cluster SMs pulls, not by rounds.)
template <int kDepth = 4>
__device__ __forceinline__ void fold_range(const float* __restrict__ part_ml, const float* __restrict__ part_acc,
                                           int b, int h, const PartIdx& pi, int first, int last, int stride, int lane,
                                           float& m, float& L, float4 (&acc)[4]) {
    for (int cc = first; cc <= last; cc += kDepth * stride) {
        float2 ml[kDepth];
        float4 a[kDepth][4];
#pragma unroll
        for (int j = 0; j < kDepth; ++j)
            if (cc + j * stride <= last) load_partial(part_ml, part_acc, b, h, pi.c(cc + j * stride), lane, ml[j], a[j]);
#pragma unroll
        for (int j = 0; j < kDepth; ++j)
            if (cc + j * stride <= last) fold_partial(ml[j], a[j], m, L, acc);
    }
}

template <int kDepth = 4>
__device__ __forceinline__ void merge_partials(const float* __restrict__ part_ml, const float* __restrict__ part_acc,
                                               int b, int h, const PartIdx& pi, int first, int last, int stride,
                                               int lane, float& m, float& L, float4 (&acc)[4]) {
    m = -INFINITY;
    L = 0.f;
#pragma unroll
    for (int k = 0; k < 4; ++k) acc[k] = make_float4(0.f, 0.f, 0.f, 0.f);
    fold_range<kDepth>(part_ml, part_acc, b, h, pi, first, last, stride, lane, m, L, acc);
}

// Address of element (row, col) of a [rows][512] bf16 matrix stored as 1024-byte
// rows whose 16-byte units are XOR-swizzled with (row & 7) (conflict-free ldmatrix).
__device__ __forceinline__ uint32_t swz1024(uint32_t base, int row, int col) {
    return base + row * 1024 + ((((col >> 3) ^ (row & 7))) << 4) + (col & 7) * 2;
}

template <int kCl, int kRq>
__device__ __forceinline__ void k3_uv_epilogue(const MlaDecodeParams& p, const uint8_t* w_s, uint32_t ahi,
                                               uint32_t alo, float* red, bool w_ok, int warp, int lane, int q, int h,
                                               int b0, int nreq, bool xmode, const ExLayout& ex, uint32_t step,
                                               __nv_bfloat16* __restrict__ out);

template <int kCl, int kRq>
__device__ __forceinline__ void k3_fused_combine(const MlaDecodeParams& p, const ExLayout& ex, uint32_t step,
                                                 int q, int h, int b0, int nreq, __nv_bfloat16* __restrict__ out);

// kFuse (peer exchange only, launched only when the whole grid is resident at
// once on every rank): after storing its lines to every rank, the CTA waits for
// the other ranks' lines of its own (requests, head, rows of v) and writes the
// combined R(out) itself, so the step needs no K4.
//
// pairs (k2_pairs): when the plan has num_ctas CTAs, the split-KV kernel ran plan
// CTAs 2k, 2k + 1 in one CTA and merged them across their boundary where it falls
// inside a request (PartIdx).
template <int kCl, int kRq, bool kFuse>
__global__ void __launch_bounds__(k3::kThreads, 1)
    k3_merge_uv(const MlaDecodeParams p, const __grid_constant__ CUtensorMap tmap_kvb, int pairs, int rpb) {
    using namespace k3;
    MLA_TL_SCOPE(2);
    using Sh = Shape<kCl, kRq>;
    constexpr int kABytes = Sh::kABytes;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* w_s = smem;
    uint8_t* a_hi = smem + Sh::kWBytes;
    uint8_t* a_lo = a_hi + kABytes;
    float* red_acc = reinterpret_cast<float*>(a_lo + kABytes);           // [kWarps][512]
    float* xch = reinterpret_cast<float*>(a_lo + kABytes + kRedBytes);     // [kCl][kRq][512 + 4]: acc, m, L
    uint64_t* bar = reinterpret_cast<uint64_t*>(a_lo + kABytes + kRedBytes + Sh::kXBytes);

    const WsLayout ws = ws_layout(p);
    const char* wsb = reinterpret_cast<const char*>(p.workspace);
    const int32_t* cum = reinterpret_cast<const int32_t*>(wsb + ws.tiles_cum);
    const float* part_ml = reinterpret_cast<const float*>(wsb + ws.part_ml);
    const float* part_acc = reinterpret_cast<const float*>(wsb + ws.part_acc);
    __nv_bfloat16* out = reinterpret_cast<__nv_bfloat16*>(p.out);

    const int q = kCl > 1 ? (int)cluster_rank() : 0;  // rank within the (head, request block) cluster
    const int h = blockIdx.x / kCl;
    const int b0 = blockIdx.y * rpb;  // rpb <= kRq requests per block (rows past them are zero)
    const int nreq = min(rpb, p.batch - b0);

    // cluster form: bar[1] counts the bytes of the other ranks' folds pushed into xch
    constexpr uint32_t kPushBytes = (kLora + 2) * 4;  // one request's acc[512], m, L
    if (threadIdx.x == 0) {  // W_UV is a weight: no kernel writes it, so it may load before pdl_wait
        mbar_init(bar, 1);
        if (kCl > 1) mbar_init(bar + 1, 1);
        fence_mbar_init();
        mbar_arrive_expect_tx(bar, Sh::kWBytes);
        tma_load_3d(w_s, &tmap_kvb, bar, 0, h * kKvbHead + kNope + q * Sh::kVRows, 0, kCacheEvictLast);
        if (kCl > 1) mbar_arrive_expect_tx(bar + 1, (uint32_t)(kCl - 1) * (uint32_t)nreq * kPushBytes);
    }
    if (kCl > 1) cluster_sync_all();  // every rank's bar[1] is initialised before any rank pushes into it
    pdl_trigger();

    // The split plan's prefix sums of this block (cum_s) and the tile total. Batches
    // of at most 64 requests derive them from the step's inputs before the wait (the
    // rule K1's planner and K2 use, plan_tiles), so the first partial loads follow the
    // wait directly; larger batches read K1's prefix sums after it.
    __shared__ int32_t cum_s[kRq + 1];
    __shared__ int32_t pre_tot[2];
    __shared__ int64_t U_s;
    constexpr int kPrePlan = 64;
    const bool pre = p.batch <= kPrePlan;
    if (pre) {
        int n = 0, incl = 0;
        if (threadIdx.x < kPrePlan) {
            n = (int)threadIdx.x < p.batch ? plan_tiles(p, threadIdx.x) : 0;
            incl = n;
            const int ln = threadIdx.x & 31;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int t = __shfl_up_sync(0xffffffffu, incl, o);
                if (ln >= o) incl += t;
            }
            if (ln == 31) pre_tot[threadIdx.x >> 5] = incl;
        }
        __syncthreads();
        if (threadIdx.x < kPrePlan) {
            const int before = (threadIdx.x >> 5) ? pre_tot[0] : 0;
            const int b = (int)threadIdx.x;  // cum[b] = before + incl - n (the total for b >= batch)
            if (b >= b0 && b <= b0 + kRq) cum_s[b - b0] = before + incl - n;
            if (b == kPrePlan - 1 && b0 + kRq >= kPrePlan) cum_s[kPrePlan - b0] = before + incl;
            if (b == 0) U_s = pre_tot[0] + pre_tot[1];
        }
    }
    // Rows of the W_UV operand past nreq are zero (shared memory only, so before the wait).
    for (int i = threadIdx.x; i < (kRq - nreq) * (kLora / 8); i += kThreads) {
        const int r = nreq + i / (kLora / 8), col = (i % (kLora / 8)) * 8;
        const uint32_t ahi0 = smem_u32(a_hi), alo0 = smem_u32(a_lo);
        *reinterpret_cast<uint4*>(a_hi + (swz1024(ahi0, r, col) - ahi0)) = make_uint4(0u, 0u, 0u, 0u);
        *reinterpret_cast<uint4*>(a_lo + (swz1024(alo0, r, col) - alo0)) = make_uint4(0u, 0u, 0u, 0u);
    }
    pdl_wait();  // partials from K2, plan from K1
    MLA_TL_WAITED(2);
    if (!pre) {
        if (threadIdx.x == 0) U_s = cum[p.batch];
        if (threadIdx.x <= kRq) cum_s[threadIdx.x] = cum[min(b0 + (int)threadIdx.x, p.batch)];
    }
    __syncthreads();
    const int64_t U = U_s;
    const int G = (int)(U < 1 ? 1 : (U < (int64_t)p.num_ctas ? U : (int64_t)p.num_ctas));
    const bool paired = pairs && G == p.num_ctas;

    // Peer exchange (p.world > 0): this step's number = steps completed + 1. The
    // counter was last written by the previous step's K4, which completed before
    // this kernel's pdl_wait returned.
    const bool xmode = p.world > 0;
    const ExLayout ex = ex_layout(p.world, p.exchange_batch);
    __shared__ uint32_t step_s;
    if (xmode && threadIdx.x == 0)
        step_s = __ldcg(reinterpret_cast<const uint32_t*>(ex_buf(p, p.rank) + ex.ctl)) + 1;

    // ---- merge: o_c[r][l] = sum_c w_c acc_c[l] / sum_c w_c l_c ----
    // Every fold visits partials in plan-CTA order; requests without tiles (invalid
    // position) get a zero o_c.
    __shared__ float red_ml[kWarps][2];
    __syncthreads();  // step_s
    const uint32_t ahi = smem_u32(a_hi), alo = smem_u32(a_lo);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    // request r's partials: n of them, at the plan CTAs pi.c(0 .. n - 1)
    auto part_range = [&](int r, PartIdx& pi, int& n) -> bool {
        if (r >= nreq || cum_s[r + 1] <= cum_s[r]) return false;  // invalid position: no tiles
        const int c0 = plan_cta_of(cum_s[r], U, G), c1 = plan_cta_of(cum_s[r + 1] - 1, U, G);
        pi = PartIdx{c0, paired};
        n = paired ? 1 + (c1 >> 1) - (c0 >> 1) : c1 - c0 + 1;
        return true;
    };
    // o_c -> bf16 hi/lo operands of request r; lane owns l = 4 lane + 128 k
    auto store_oc = [&](int r, const float4 (&acc)[4], float inv_L) {
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
    };
    auto store_ml = [&](int r, float m, float L) {
        if (r >= nreq || lane != 0 || q != 0) return;
        if (xmode) {  // into slot p.rank of every rank's exchange buffer
#pragma unroll
            for (int d = 0; d < kMaxRanks; ++d) {
                if (d >= p.world) break;
                st_line(ex_lines(ex_buf(p, d), ex, p.world, p.exchange_batch, step_s & 1u, p.rank, b0 + r, h) + kV / 2,
                        m, L, step_s);
            }
        } else if (p.shard_out) {
            float* so = p.shard_out + ((int64_t)(b0 + r) * kHeads + h) * MLA_SHARD_STRIDE;
            so[kV] = m;
            so[kV + 1] = L;
        }
    };
    // this CTA's fold of request r: finished here (kCl = 1), or published for the cluster
    auto publish = [&](int r, float m, float L, const float4 (&acc)[4]) {
        if (kCl == 1) {
            store_ml(r, m, L);
            store_oc(r, acc, L > 0.f ? 1.f / L : 0.f);
        } else {  // into slot [q][r] of xch in this CTA and in every other rank of the cluster
            float* x = xch + (q * kRq + r) * (kLora + 4);
#pragma unroll
            for (int k = 0; k < 4; ++k) *reinterpret_cast<float4*>(x + 4 * lane + 128 * k) = acc[k];
            if (lane == 0) { x[kLora] = m; x[kLora + 1] = L; }
            const uint32_t xl = smem_u32(x), bl = smem_u32(bar + 1);
#pragma unroll
            for (int c = 0; c < kCl; ++c) {
                if (c == q) continue;
                const uint32_t xr = dsmem_addr(xl, (uint32_t)c), br = dsmem_addr(bl, (uint32_t)c);
#pragma unroll
                for (int k = 0; k < 4; ++k) dsmem_push4(xr + (uint32_t)(4 * lane + 128 * k) * 4u, acc[k], br);
                if (lane == 0) dsmem_push2(xr + (uint32_t)kLora * 4u, make_float2(m, L), br);
            }
        }
    };

    // Warps per request: the largest power of two <= 8 / nreq (8 for one request,
    // 1 for 5 or more). A group of wpr warps of cluster rank q folds request r's
    // partials c0 + q + kCl wi, c0 + q + kCl (wi + wpr), ... (wi = warp within the
    // group), then the group's warp results are combined through shared memory in
    // warp order.
    const int wpr = nreq == 1 ? 8 : nreq == 2 ? 4 : nreq <= 4 ? 2 : 1;
    const int groups = kWarps / wpr, gi = warp / wpr, wi = warp % wpr;
    const int iters = (nreq + groups - 1) / groups;
    if (wpr == 1) {
        // One warp per request (5 or more requests): two requests per pass, the first
        // two partials of both loaded together, so that a warp's requests do not each
        // wait for their own round trip in turn. Each request still folds its partials
        // in plan order. (Three per request measured the same: the merge is bound by
        // the L2 lines an SM keeps in flight, ~30 GB/s per SM, not by round trips.)
        const int first = q, stride = kCl;
#pragma unroll 1
        for (int it = 0; it < iters; it += 2) {
            int r2[2], n2[2] = {0, 0};
            PartIdx pi[2] = {{0, false}, {0, false}};
            bool v[2];
            float2 ml[2][2];
            float4 a[2][2][4];
#pragma unroll
            for (int x = 0; x < 2; ++x) {
                r2[x] = gi + (it + x) * groups;
                v[x] = it + x < iters && part_range(r2[x], pi[x], n2[x]) && first < n2[x];
#pragma unroll
                for (int j = 0; j < 2; ++j)
                    if (v[x] && first + j * stride < n2[x])
                        load_partial(part_ml, part_acc, b0 + r2[x], h, pi[x].c(first + j * stride), lane, ml[x][j],
                                     a[x][j]);
            }
#pragma unroll
            for (int x = 0; x < 2; ++x) {
                float m = -INFINITY, L = 0.f;
                float4 acc[4];
#pragma unroll
                for (int k = 0; k < 4; ++k) acc[k] = make_float4(0.f, 0.f, 0.f, 0.f);
                if (v[x]) {
#pragma unroll
                    for (int j = 0; j < 2; ++j)
                        if (first + j * stride < n2[x]) fold_partial(ml[x][j], a[x][j], m, L, acc);
                    fold_range(part_ml, part_acc, b0 + r2[x], h, pi[x], first + 2 * stride, n2[x] - 1, stride, lane,
                               m, L, acc);
                }
                if (r2[x] < nreq && it + x < iters) publish(r2[x], m, L, acc);
            }
        }
    } else {
#pragma unroll 1
    for (int it = 0; it < iters; ++it) {  // uniform trip count: the barriers below are CTA-wide
        const int r = gi + it * groups;
        PartIdx pi{0, false};
        int n = 0;
        float4 acc[4];
        float m = -INFINITY, L = 0.f;
        const int first = q + kCl * wi;
        if (part_range(r, pi, n) && first < n)
            merge_partials(part_ml, part_acc, b0 + r, h, pi, first, n - 1, kCl * wpr, lane, m, L, acc);
        else
            for (int k = 0; k < 4; ++k) acc[k] = make_float4(0.f, 0.f, 0.f, 0.f);
        if (lane == 0) { red_ml[warp][0] = m; red_ml[warp][1] = L; }
#pragma unroll
        for (int k = 0; k < 4; ++k)
            *reinterpret_cast<float4*>(red_acc + warp * kLora + 4 * lane + 128 * k) = acc[k];
        __syncthreads();
        if (wi == 0 && r < nreq) {
            const int w0 = warp;
            float gm = -INFINITY;
            for (int v = 0; v < wpr; ++v)
                if (red_ml[w0 + v][1] > 0.f) gm = fmaxf(gm, red_ml[w0 + v][0]);
            float Lt = 0.f;
            float4 tot[4];
#pragma unroll
            for (int k = 0; k < 4; ++k) tot[k] = make_float4(0.f, 0.f, 0.f, 0.f);
            for (int v = 0; v < wpr; ++v) {
                const float wv = red_ml[w0 + v][1] > 0.f ? exp2f(red_ml[w0 + v][0] - gm) : 0.f;
                Lt = fmaf(wv, red_ml[w0 + v][1], Lt);
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    const float4 x = *reinterpret_cast<const float4*>(red_acc + (w0 + v) * kLora + 4 * lane + 128 * k);
                    tot[k].x = fmaf(wv, x.x, tot[k].x); tot[k].y = fmaf(wv, x.y, tot[k].y);
                    tot[k].z = fmaf(wv, x.z, tot[k].z); tot[k].w = fmaf(wv, x.w, tot[k].w);
                }
            }
            publish(r, gm, Lt, tot);
        }
        __syncthreads();
    }

    }
    if (kCl > 1) {
        // The cluster's kCl folds of each request, combined in rank order: every CTA
        // holds all ranks' (acc, m, L) in its own xch once the other ranks' pushes have
        // landed (bar[1]), so each has the whole o_c for its slice of W_UV. Warp w
        // combines requests w and w + 8.
        __syncthreads();  // this CTA's own slot, written by its warps
        MLA_TL_MARK(2, 4);
        {
            int dummy = 0;
            if (!mbar_wait(bar + 1, 0, &dummy, err_sink(p))) return;
        }
#pragma unroll 1
        for (int rr = 0; rr < 2; ++rr) {
            const int r = warp + kWarps * rr;
            if (r >= nreq) continue;
            float2 ml[kCl];
            float4 xs[kCl][4];
#pragma unroll
            for (int c = 0; c < kCl; ++c) {
                const float* x = xch + (c * kRq + r) * (kLora + 4);
                ml[c] = make_float2(x[kLora], x[kLora + 1]);
#pragma unroll
                for (int k = 0; k < 4; ++k) xs[c][k] = *reinterpret_cast<const float4*>(x + 4 * lane + 128 * k);
            }
            float gm = -INFINITY;
#pragma unroll
            for (int c = 0; c < kCl; ++c)
                if (ml[c].y > 0.f) gm = fmaxf(gm, ml[c].x);
            float Lt = 0.f;
            float4 tot[4];
#pragma unroll
            for (int k = 0; k < 4; ++k) tot[k] = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
            for (int c = 0; c < kCl; ++c) {
                const float wv = ml[c].y > 0.f ? exp2f(ml[c].x - gm) : 0.f;
                Lt = fmaf(wv, ml[c].y, Lt);
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    const float4 x = xs[c][k];
                    tot[k].x = fmaf(wv, x.x, tot[k].x); tot[k].y = fmaf(wv, x.y, tot[k].y);
                    tot[k].z = fmaf(wv, x.z, tot[k].z); tot[k].w = fmaf(wv, x.w, tot[k].w);
                }
            }
            store_ml(r, gm, Lt);
            store_oc(r, tot, Lt > 0.f ? 1.f / Lt : 0.f);
        }
    }
    __syncthreads();
    MLA_TL_MARK(2, 5);  // merge done
    bool w_ok;
    {
        int dummy = 0;
        w_ok = mbar_wait(bar, 0, &dummy, err_sink(p));
    }
    if (kCl == 1) MLA_TL_MARK(2, 4);  // W_UV staged (the cluster form marks its published folds)

    // ---- out[r][v] = sum_l o_c[r][l] W_UV[h][v][l] for this CTA's kVRows rows of v;
    // warp w owns v in [16w, 16w+16) ----
    if (!kFuse) {
        k3_uv_epilogue<kCl, kRq>(p, w_s, ahi, alo, red_acc, w_ok, warp, lane, q, h, b0, nreq, xmode, ex,
                                 xmode ? step_s : 0u, out);
        return;
    }
    k3_uv_epilogue<kCl, kRq>(p, w_s, ahi, alo, red_acc, w_ok, warp, lane, q, h, b0, nreq, true, ex, step_s, out);
    k3_fused_combine<kCl, kRq>(p, ex, step_s, q, h, b0, nreq, out);
    if (threadIdx.x == 0) {  // the last CTA to finish (every CTA's thread 0 has read the counter) advances it
        uint32_t* ctl = reinterpret_cast<uint32_t*>(ex_buf(p, p.rank) + ex.ctl);
        __threadfence();
        if (atomicAdd(ctl + 1, 1u) == gridDim.x * gridDim.y - 1) {
            ctl[1] = 0;
            __threadfence();
            atomicExch(ctl, step_s);
        }
    }
}

// The combine of a fused K3 CTA: for each of its requests and line pairs of v, the
// rank-ordered fold of combine_head over the world shards' lines (this rank's own
// included), polled until they carry this step (bounded by exchange_timeout_us; on
// timeout MLA_DEV_PEER_TIMEOUT and zeros). One line (two values of v) per task.
template <int kCl, int kRq>
__device__ __forceinline__ void k3_fused_combine(const MlaDecodeParams& p, const ExLayout& ex, uint32_t step,
                                                 int q, int h, int b0, int nreq, __nv_bfloat16* __restrict__ out) {
    using Sh = k3::Shape<kCl, kRq>;
    constexpr int kLines = Sh::kVRows / 2;  // lines of this CTA's rows of v, per request
    char* own = ex_buf(p, p.rank);
    const uint64_t limit_ns = (uint64_t)(p.exchange_timeout_us > 0 ? p.exchange_timeout_us : 2000000) * 1000ull;
    const uint64_t t0 = globaltimer_ns();
    bool ok = true;
    for (int task = threadIdx.x; task < nreq * kLines; task += k3::kThreads) {
        const int b = b0 + task / kLines;
        const int line = q * kLines + task % kLines;  // v = 2 line, 2 line + 1
        // every shard's (m, L) line and y line, loaded together, then waited on
        const ulonglong2* base[kMaxRanks];
        ulonglong2 mlv[kMaxRanks], yv[kMaxRanks];
#pragma unroll
        for (int r = 0; r < kMaxRanks; ++r) {
            if (r >= p.world) break;
            base[r] = ex_lines(own, ex, p.world, p.exchange_batch, step & 1u, r, b, h);
            mlv[r] = ld_line(base[r] + kV / 2);
            yv[r] = ld_line(base[r] + line);
        }
        float gm = -INFINITY;
#pragma unroll
        for (int r = 0; r < kMaxRanks; ++r) {
            if (r >= p.world) break;
            if (ok) ok = wait_line(base[r] + kV / 2, step, mlv[r], t0, limit_ns) &&
                         wait_line(base[r] + line, step, yv[r], t0, limit_ns);
            gm = fmaxf(gm, line_lo(mlv[r]));
        }
        float a0 = 0.f, a1 = 0.f, W = 0.f;
#pragma unroll
        for (int r = 0; r < kMaxRanks; ++r) {
            if (r >= p.world || !ok) break;
            const float Lr = line_hi(mlv[r]);
            if (!(Lr > 0.f)) continue;  // an empty shard contributes nothing
            const float w = Lr * exp2f(line_lo(mlv[r]) - gm);
            W += w;
            a0 = fmaf(w, line_lo(yv[r]), a0);
            a1 = fmaf(w, line_hi(yv[r]), a1);
        }
        const float inv = W > 0.f ? 1.f / W : 0.f;
        // after a timeout the remaining tasks poll nothing and write zeros
        *reinterpret_cast<uint32_t*>(out + (int64_t)b * p.out_stride + h * kV + 2 * line) =
            ok ? pack_bf16(a0 * inv, a1 * inv) : 0u;
    }
    if (!ok) record_error(err_sink(p), MLA_DEV_PEER_TIMEOUT);
}

// The W_UV MMA and its epilogue, by all eight warps of a K3 CTA: warp w takes the
// 16 rows of v of group w % kGroups over the 512 / kKp latent columns of part
// w / kGroups, for all kRq requests (kRq / 16 m16 tiles); the hi and lo halves of
// o_c accumulate separately (independent MMA chains). The plain form's 128 rows
// give every warp its own group (kKp = 1). The cluster form's 32 rows are two
// groups, so its warps split the latent columns four ways: the parts meet in
// shared memory (red, the merge's reduction area, free by now) in part order. The
// part-0 warps write R(out) in bf16, or the fp32 shard partial y (into shard_out,
// or in exchange mode into slot p.rank of every rank's exchange buffer). (Splitting
// the plain form into 4 groups x 2 parts of 32 rows measured 1.5 us slower at 32
// requests.) !w_ok (the W_UV load gave up): every warp still meets any barrier,
// and nothing is written.
template <int kCl, int kRq>
struct UvSplit {
    static constexpr int kVRows = k3::Shape<kCl, kRq>::kVRows;
    static constexpr int kVg = 16;                            // rows of v per warp
    static constexpr int kGroups = kVRows / kVg;              // v groups
    static constexpr int kKp = k3::kWarps / kGroups;          // latent parts
    static constexpr int kKs = kLora / 16 / kKp;              // k-steps of 16 per part
    static constexpr int kNt = kVg / 8;                       // n8 tiles per warp
    static constexpr int kFrag = k3::Shape<kCl, kRq>::kMt * kNt * 4;  // accumulators per lane
    static_assert(kGroups * kKp == k3::kWarps && kKs * kKp * 16 == kLora, "warps = v groups x latent parts");
    static_assert((kKp - 1) * kGroups * kFrag * 32 * 4 <= k3::kRedBytes, "part sums fit the reduction area");
};

template <int kCl, int kRq>
__device__ __forceinline__ void k3_uv_epilogue(const MlaDecodeParams& p, const uint8_t* w_s, uint32_t ahi,
                                               uint32_t alo, float* red, bool w_ok, int warp, int lane, int q, int h,
                                               int b0, int nreq, bool xmode, const ExLayout& ex, uint32_t step,
                                               __nv_bfloat16* __restrict__ out) {
    using Sh = k3::Shape<kCl, kRq>;
    using Sp = UvSplit<kCl, kRq>;
    constexpr int kMt = Sh::kMt, kNt = Sp::kNt;
    const int g = lane >> 2, t4 = lane & 3, m8 = lane >> 3, r8 = lane & 7;
    const int vg = warp % Sp::kGroups, kp = warp / Sp::kGroups;
    const uint32_t wb = smem_u32(w_s);
    float acc[kMt][kNt][4], acl[kMt][kNt][4];
#pragma unroll
    for (int mt = 0; mt < kMt; ++mt)
#pragma unroll
        for (int n = 0; n < kNt; ++n)
#pragma unroll
            for (int e = 0; e < 4; ++e) acc[mt][n][e] = acl[mt][n][e] = 0.f;
#pragma unroll 4
    for (int kk = 0; kk < Sp::kKs; ++kk) {
        const int ks = kp * Sp::kKs + kk;
        uint32_t bf[kNt][2];  // B fragments of this warp's n8 tiles of v
#pragma unroll
        for (int np = 0; np < kNt / 2; ++np) {
            const int v = Sp::kVg * vg + 16 * np + (m8 >> 1) * 8 + r8;
            const int l = 16 * ks + (m8 & 1) * 8;
            ldsm_x4(wb + (l >> 6) * (Sh::kVRows * 128) + v * 128 + ((((l & 63) >> 3) ^ r8) << 4), bf[2 * np][0],
                    bf[2 * np][1], bf[2 * np + 1][0], bf[2 * np + 1][1]);
        }
#pragma unroll
        for (int mt = 0; mt < kMt; ++mt) {
            uint32_t ah[4], al[4];
            const int row = 16 * mt + (m8 & 1) * 8 + r8, col = 16 * ks + (m8 >> 1) * 8;
            ldsm_x4(swz1024(ahi, row, col), ah[0], ah[1], ah[2], ah[3]);
            ldsm_x4(swz1024(alo, row, col), al[0], al[1], al[2], al[3]);
#pragma unroll
            for (int n = 0; n < kNt; ++n) {
                mma16816(acc[mt][n], ah, bf[n][0], bf[n][1]);
                mma16816(acl[mt][n], al, bf[n][0], bf[n][1]);
            }
        }
    }
#pragma unroll
    for (int mt = 0; mt < kMt; ++mt)
#pragma unroll
        for (int n = 0; n < kNt; ++n)
#pragma unroll
            for (int e = 0; e < 4; ++e) acc[mt][n][e] += acl[mt][n][e];
    if (Sp::kKp > 1) {  // part sums of parts 1.. -> red, added by the part-0 warp of the group in part order
        float4* slot = reinterpret_cast<float4*>(red) + (size_t)((kp - 1) * Sp::kGroups + vg) * (Sp::kFrag / 4) * 32;
        if (kp > 0) {
#pragma unroll
            for (int mt = 0; mt < kMt; ++mt)
#pragma unroll
                for (int n = 0; n < kNt; ++n)
                    slot[(mt * kNt + n) * 32 + lane] = make_float4(acc[mt][n][0], acc[mt][n][1], acc[mt][n][2],
                                                                   acc[mt][n][3]);
        }
        __syncthreads();
        if (kp > 0) return;
#pragma unroll 1
        for (int k2 = 1; k2 < Sp::kKp; ++k2) {
            const float4* src = reinterpret_cast<const float4*>(red) + (size_t)((k2 - 1) * Sp::kGroups + vg) *
                                                                        (Sp::kFrag / 4) * 32;
#pragma unroll
            for (int mt = 0; mt < kMt; ++mt)
#pragma unroll
                for (int n = 0; n < kNt; ++n) {
                    const float4 x = src[(mt * kNt + n) * 32 + lane];
                    acc[mt][n][0] += x.x; acc[mt][n][1] += x.y; acc[mt][n][2] += x.z; acc[mt][n][3] += x.w;
                }
        }
    }
    if (!w_ok) return;
    // The thread holds v, v + 1 of requests 16 mt + g (acc[..][0..1]) and 16 mt + g + 8 (acc[..][2..3]).
    const int v_base = q * Sh::kVRows;
#pragma unroll
    for (int mt = 0; mt < kMt; ++mt)
#pragma unroll
        for (int n = 0; n < kNt; ++n)
#pragma unroll
            for (int hf = 0; hf < 2; ++hf) {
                const int r = 16 * mt + g + 8 * hf;
                if (r >= nreq) continue;
                const int v = v_base + Sp::kVg * vg + 8 * n + 2 * t4;
                const float y0 = acc[mt][n][2 * hf], y1 = acc[mt][n][2 * hf + 1];
                if (xmode) {  // fp32 y = W_UV o_c / L of this shard, to every rank
#pragma unroll
                    for (int d = 0; d < kMaxRanks; ++d) {
                        if (d >= p.world) break;
                        st_line(ex_lines(ex_buf(p, d), ex, p.world, p.exchange_batch, step & 1u, p.rank, b0 + r, h) +
                                    v / 2,
                                y0, y1, step);
                    }
                } else if (p.shard_out) {  // sequence-sharded step: fp32 y = W_UV o_c / L of this shard
                    *reinterpret_cast<float2*>(p.shard_out + ((int64_t)(b0 + r) * kHeads + h) * MLA_SHARD_STRIDE + v) =
                        make_float2(y0, y1);
                } else {
                    *reinterpret_cast<uint32_t*>(out + (int64_t)(b0 + r) * p.out_stride + h * kV + v) =
                        pack_bf16(y0, y1);
                }
            }
}

// Cross-shard combine of one (request, head): out[128h + v] = bf16( sum_r w_r y_r[v] /
// sum_r w_r ), w_r = L_r 2^(m_r - max m), shards r = 0, 1, ... folded in order from
// base + r * shard_stride. kPeerData: the partials were written by other GPUs during
// this kernel's lifetime, so they are read from L2 (ld.global.cg), not through L1.
template <bool kPeerData>
__device__ __forceinline__ void combine_head(const float* __restrict__ base, int64_t shard_stride, int n_shards,
                                             int v0, __nv_bfloat16* __restrict__ o) {
    auto ld1 = [](const float* a) -> float { return kPeerData ? __ldcg(a) : *a; };
    auto ld4 = [](const float* a) -> float4 {
        return kPeerData ? __ldcg(reinterpret_cast<const float4*>(a)) : *reinterpret_cast<const float4*>(a);
    };
    float gm = -INFINITY;
    for (int r = 0; r < n_shards; ++r) gm = fmaxf(gm, ld1(base + r * shard_stride + kV));
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    float W = 0.f;
    for (int r = 0; r < n_shards; ++r) {
        const float* pr = base + r * shard_stride;
        const float Lr = ld1(pr + kV + 1);
        if (!(Lr > 0.f)) continue;  // an empty shard contributes nothing
        const float w = Lr * exp2f(ld1(pr + kV) - gm);
        W += w;
        const float4 y0 = ld4(pr + v0);
        const float4 y1 = ld4(pr + v0 + 4);
        acc[0] = fmaf(w, y0.x, acc[0]); acc[1] = fmaf(w, y0.y, acc[1]);
        acc[2] = fmaf(w, y0.z, acc[2]); acc[3] = fmaf(w, y0.w, acc[3]);
        acc[4] = fmaf(w, y1.x, acc[4]); acc[5] = fmaf(w, y1.y, acc[5]);
        acc[6] = fmaf(w, y1.z, acc[6]); acc[7] = fmaf(w, y1.w, acc[7]);
    }
    const float inv = W > 0.f ? 1.f / W : 0.f;
#pragma unroll
    for (int k = 0; k < 8; k += 2)
        *reinterpret_cast<uint32_t*>(o + k) = pack_bf16(acc[k] * inv, acc[k + 1] * inv);
}

// Cross-shard combine of a sequence-sharded step whose partials were gathered by
// the caller (parts [n_shards][batch][16][132]). Block = request, thread = (head,
// 8 values of v).
__global__ void __launch_bounds__(256) k4_combine_shards(const float* __restrict__ parts, int n_shards, int batch,
                                                         __nv_bfloat16* __restrict__ out, int64_t out_stride) {
    const int b = blockIdx.x;
    const int h = threadIdx.x >> 4, v0 = (threadIdx.x & 15) * 8;
    combine_head<false>(parts + ((int64_t)b * kHeads + h) * MLA_SHARD_STRIDE,
                        (int64_t)batch * kHeads * MLA_SHARD_STRIDE, n_shards, v0,
                        out + (int64_t)b * out_stride + h * kV + v0);
}

// K4 of the peer exchange: the combine of combine_head, over the shard partials
// every rank's K3 stored into this rank's exchange buffer as step-tagged lines.
// Block = request, thread = (head, 8 values of v). Each thread polls the lines it
// needs until they carry this step's number (bounded by exchange_timeout_us; on
// timeout the block records MLA_DEV_PEER_TIMEOUT and writes zeros). The last block
// to finish advances the buffer's step counter.
template <int kW>  // an upper bound on p.world (2, 4 or 8): sizes the per-thread line arrays
__global__ void __launch_bounds__(256) k4_exchange_combine(const MlaDecodeParams p) {
    MLA_TL_SCOPE(3);
    const int b = blockIdx.x;
    const int h = threadIdx.x >> 4, v0 = (threadIdx.x & 15) * 8;
    pdl_trigger();
    pdl_wait();  // this rank's K3 has completed (and read the step counter)
    MLA_TL_WAITED(3);
    const ExLayout ex = ex_layout(p.world, p.exchange_batch);
    char* own = ex_buf(p, p.rank);
    uint32_t* ctl = reinterpret_cast<uint32_t*>(own + ex.ctl);
    __shared__ uint32_t step_s;
    __shared__ int fail_s;
    if (threadIdx.x == 0) {
        step_s = __ldcg(ctl) + 1;
        fail_s = 0;
    }
    __syncthreads();
    const uint32_t step = step_s;
    const uint64_t limit_ns = (uint64_t)(p.exchange_timeout_us > 0 ? p.exchange_timeout_us : 2000000) * 1000ull;
    const uint64_t t0 = globaltimer_ns();
    bool ok = true;
    // every shard's (m, L) line and the four y lines of this thread, loaded together,
    // then waited on
    const ulonglong2* base[kW];
    ulonglong2 mlv[kW], yv[kW][4];
#pragma unroll
    for (int r = 0; r < kW; ++r) {
        if (r >= p.world) break;
        base[r] = ex_lines(own, ex, p.world, p.exchange_batch, step & 1u, r, b, h);
        mlv[r] = ld_line(base[r] + kV / 2);
#pragma unroll
        for (int k = 0; k < 4; ++k) yv[r][k] = ld_line(base[r] + v0 / 2 + k);
    }
    float gm = -INFINITY;
#pragma unroll
    for (int r = 0; r < kW; ++r) {
        if (r >= p.world) break;
        if (ok) ok = wait_line(base[r] + kV / 2, step, mlv[r], t0, limit_ns);
#pragma unroll
        for (int k = 0; k < 4; ++k)
            if (ok) ok = wait_line(base[r] + v0 / 2 + k, step, yv[r][k], t0, limit_ns);
        gm = fmaxf(gm, line_lo(mlv[r]));
    }
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    float W = 0.f;
#pragma unroll
    for (int r = 0; r < kW; ++r) {
        if (r >= p.world || !ok) break;
        const float Lr = line_hi(mlv[r]);
        if (!(Lr > 0.f)) continue;  // an empty shard contributes nothing
        const float w = Lr * exp2f(line_lo(mlv[r]) - gm);
        W += w;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            acc[2 * k] = fmaf(w, line_lo(yv[r][k]), acc[2 * k]);
            acc[2 * k + 1] = fmaf(w, line_hi(yv[r][k]), acc[2 * k + 1]);
        }
    }
    if (!ok) {
        record_error(err_sink(p), MLA_DEV_PEER_TIMEOUT);
        fail_s = 1;
    }
    __syncthreads();
    __nv_bfloat16* o = reinterpret_cast<__nv_bfloat16*>(p.out) + (int64_t)b * p.out_stride + h * kV + v0;
    const float inv = W > 0.f ? 1.f / W : 0.f;
#pragma unroll
    for (int k = 0; k < 8; k += 2)
        *reinterpret_cast<uint32_t*>(o + k) = fail_s ? 0u : pack_bf16(acc[k] * inv, acc[k + 1] * inv);
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence();
        if (atomicAdd(ctl + 1, 1u) == gridDim.x - 1) {  // every block has read the counter
            ctl[1] = 0;
            __threadfence();
            atomicExch(ctl, step);
        }
    }
}

cudaError_t launch_exchange_combine(const MlaDecodeParams& p, cudaStream_t stream) {
    if (p.world <= 2) return launch_pdl(k4_exchange_combine<2>, dim3(p.batch), dim3(256), 0, stream, p);
    if (p.world <= 4) return launch_pdl(k4_exchange_combine<4>, dim3(p.batch), dim3(256), 0, stream, p);
    return launch_pdl(k4_exchange_combine<kMaxRanks>, dim3(p.batch), dim3(256), 0, stream, p);
}

cudaError_t launch_combine_shards(const float* parts, int n_shards, int batch, void* out, int64_t out_stride,
                                  cudaStream_t stream) {
    k4_combine_shards<<<batch, 256, 0, stream>>>(parts, n_shards, batch, reinterpret_cast<__nv_bfloat16*>(out),
                                                out_stride);
    return cudaGetLastError();
}

template <int kCl, int kRq, bool kFuse>
static cudaError_t k3_set_smem() {
    return cudaFuncSetAttribute(k3_merge_uv<kCl, kRq, kFuse>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                k3::Shape<kCl, kRq>::kSmemBytes);
}

cudaError_t k3_configure() {
    constexpr int kCl = k3::kClusterCtas, kR = k3::kReq;
    cudaError_t e;
    if ((e = k3_set_smem<1, kR, false>()) != cudaSuccess || (e = k3_set_smem<1, kR, true>()) != cudaSuccess ||
        (e = k3_set_smem<1, 2 * kR, false>()) != cudaSuccess || (e = k3_set_smem<1, 2 * kR, true>()) != cudaSuccess ||
        (e = k3_set_smem<kCl, kR, false>()) != cudaSuccess || (e = k3_set_smem<kCl, kR, true>()) != cudaSuccess)
        return e;
    return cudaSuccess;
}

// Rows of W_UV per CTA of the launch chosen by launch_merge_uv (its TMA box height).
int k3_w_rows(int batch) { return k3_use_cluster(batch) ? k3::Shape<k3::kClusterCtas>::kVRows : kV; }

namespace {

// The K3 launch for a batch: cluster form (4 CTAs per (head, 16 requests)) for
// batches of at most 4 blocks of 16; else the plain form in blocks of 16 while 16
// heads x blocks fill at most one wave of SMs (one CTA per SM: W_UV[h] is 128 KB of
// shared memory), beyond that in blocks of 32 (two m16 tiles on one staged W_UV[h]),
// which halves the waves.
struct K3Launch {
    int cl, rq, rpb;  // form, m16 capacity of a block, requests per block
    dim3 grid;
};

// The cluster form fills two blocks where the batch allows: 5-8 requests run as two
// blocks of 4 and 9-16 as two of 8 (128 CTAs instead of 64), so each CTA folds half
// as many partials; the W_UV MMA still runs one m16 tile, its rows past the block zero.
inline int k3_cluster_rpb(int batch) { return batch <= 4 ? 4 : batch <= 8 ? 4 : batch <= 16 ? 8 : k3::kReq; }

K3Launch k3_launch(int batch, int sm_count) {
    if (k3_use_cluster(batch)) {
        const int rpb = k3_cluster_rpb(batch);
        return {k3::kClusterCtas, k3::kReq, rpb, dim3(kHeads * k3::kClusterCtas, (batch + rpb - 1) / rpb)};
    }
    const int blocks16 = (batch + k3::kReq - 1) / k3::kReq;
    if (kHeads * blocks16 <= sm_count) return {1, k3::kReq, k3::kReq, dim3(kHeads, blocks16)};
    return {1, 2 * k3::kReq, 2 * k3::kReq, dim3(kHeads, (batch + 2 * k3::kReq - 1) / (2 * k3::kReq))};
}

template <int kCl, int kRq, bool kFuse>
cudaError_t k3_launch_form(const MlaDecodeParams& p, const CUtensorMap& tmap_kvb, dim3 grid, int pairs, int rpb,
                           cudaStream_t stream, bool query_only, bool* resident) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = dim3(k3::kThreads);
    cfg.dynamicSmemBytes = k3::Shape<kCl, kRq>::kSmemBytes;
    cfg.stream = stream;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = kCl;
    attr[1].val.clusterDim.y = 1;
    attr[1].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = kCl > 1 ? 2 : 1;
    if (query_only) {  // can every CTA (cluster) of the grid be resident at once?
        int n = 0;
        cudaError_t e;
        if (kCl > 1) {
            e = cudaOccupancyMaxActiveClusters(&n, k3_merge_uv<kCl, kRq, kFuse>, &cfg);
            *resident = e == cudaSuccess && (int64_t)n * kCl >= (int64_t)grid.x * grid.y;
        } else {
            e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, k3_merge_uv<kCl, kRq, kFuse>, k3::kThreads,
                                                              k3::Shape<kCl, kRq>::kSmemBytes);
            int dev = 0, sms = 0;
            if (e == cudaSuccess) e = cudaGetDevice(&dev);
            if (e == cudaSuccess) e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
            *resident = e == cudaSuccess && (int64_t)n * sms >= (int64_t)grid.x * grid.y;
        }
        return e;
    }
    return cudaLaunchKernelEx(&cfg, k3_merge_uv<kCl, kRq, kFuse>, p, tmap_kvb, pairs, rpb);
}

template <bool kFuse>
cudaError_t k3_dispatch(const MlaDecodeParams& p, const CUtensorMap& tmap_kvb, const K3Launch& l, int pairs,
                        cudaStream_t stream, bool query_only, bool* resident) {
    if (l.cl > 1)
        return k3_launch_form<k3::kClusterCtas, k3::kReq, kFuse>(p, tmap_kvb, l.grid, pairs, l.rpb, stream,
                                                                query_only, resident);
    if (l.rq == k3::kReq)
        return k3_launch_form<1, k3::kReq, kFuse>(p, tmap_kvb, l.grid, pairs, l.rpb, stream, query_only, resident);
    return k3_launch_form<1, 2 * k3::kReq, kFuse>(p, tmap_kvb, l.grid, pairs, l.rpb, stream, query_only, resident);
}

}  // namespace

// Whether the fused K3 (exchange and combine in the same kernel) may run for this
// batch: every CTA of its grid must be resident at the same time, since each one
// waits for the same CTA of the other ranks. Pure host query.
bool k3_fused_fits(int batch, int sm_count) {
    const K3Launch l = k3_launch(batch, sm_count);
    bool resident = false;
    MlaDecodeParams dummy{};
    CUtensorMap t{};
    return k3_dispatch<true>(dummy, t, l, 0, nullptr, true, &resident) == cudaSuccess && resident;
}

cudaError_t launch_merge_uv(const MlaDecodeParams& p, const CUtensorMap& tmap_kvb, int sm_count, bool fused,
                            cudaStream_t stream) {
    const K3Launch l = k3_launch(p.batch, sm_count);
    const int pairs = k2_pairs(p, sm_count) ? 1 : 0;  // as the split-KV kernel of these params ran
    return fused ? k3_dispatch<true>(p, tmap_kvb, l, pairs, stream, false, nullptr)
                 : k3_dispatch<false>(p, tmap_kvb, l, pairs, stream, false, nullptr);
}

}  // namespace mla
