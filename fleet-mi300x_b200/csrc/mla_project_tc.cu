// The two projections around the attention task for batches beyond the weight
// stream's 64 requests, on the 5th-generation tensor cores:
//   K0: q | kv_a = R(x_n [W_q; W_kv_a]^T)             (reference_decode.py:225-231)
//   K5: h' = R(h + R(R(out) W_o^T))                    (reference_decode.py:256, 300)
// y[b][n] = epi(sum_k x[b][k] W[n][k]) over K = 2048, for N = 3648 (K0) or 2048
// (K5) weight rows. At 64 requests or fewer the weight is the whole cost and the
// weight-stream kernel (mla_project.cu) runs instead; beyond that the product is
// a GEMM (3.8 GFLOP at 256 requests for K0) with M = batch.
//
// Tiling: a CTA owns 256 batch rows (two M = 128 tcgen05 tiles) x 128 weight rows
// (N = 128) over one quarter of K (512). The four quarters of an output tile are
// the four CTAs of a thread-block cluster, so 116 CTAs cover K0 at 256 requests.
//   * warp 0, one thread: TMA producer. Per 64-column chunk of K, one box of x
//     (256 rows, rows past the batch read as zeros) and one of W (128 rows, rows
//     past N as zeros), 48 KB, into a 4-stage ring; the first four W chunks are
//     requested before the wait on the previous kernel (no kernel writes a weight).
//     No multicast.
//   * warp 1: allocates 256 columns of tensor memory (D of the two M tiles, fp32)
//     and one thread issues tcgen05.mma (kind::f16, bf16 operands, both K-major in
//     128-byte swizzled tiles), 4 K-steps x 2 M tiles per chunk, commits each
//     stage back to the producer and the last one to the epilogue.
//   * all 4 warps, epilogue: warp w reads its 32 lanes (batch rows) of D. The four
//     K-quarter partials meet through distributed shared memory: rank r of the
//     cluster sums output columns [32 r, 32 r + 32) of the tile. Each rank first
//     tells every peer that its stage ring is free (one 4-byte st.async per peer
//     on the peer's mbarrier), waits for the same from all peers, then pushes each
//     peer its 32 columns of every row (st.async, completing bytes on the peer's
//     receive mbarrier) and keeps its own. Once all three peers' bytes have landed
//     it adds the four partials in rank order (a fixed order: the result does not
//     depend on timing), rounds (and for K5 adds the residual), and stores bf16.
// Every wait is bounded (mla::mbar_wait); the protocol runs to its end on every
// rank even after a timeout, which is recorded in the error word.
#include <cuda.h>

#include "mla_common.cuh"
#include "mla_mma.cuh"
#include "mla_tiles.cuh"

namespace mla {

namespace k0w {
constexpr int kBM = 256;                          // batch rows per CTA: two M = 128 MMA tiles
constexpr int kBN = 128;                          // weight rows per CTA: the MMA's N
constexpr int kSplit = 4;                         // K quarters = CTAs of a cluster
constexpr int kKc = 64;                           // K per chunk: one 128-byte swizzle atom of bf16
constexpr int kChunks = kHidden / kSplit / kKc;   // 8
constexpr int kStages = 4;
constexpr int kABytes = kBM * kKc * 2;            // 32768: [256 rows][128 B]
constexpr int kBBytes = kBN * kKc * 2;            // 16384: [128 rows][128 B]
constexpr int kStageBytes = kABytes + kBBytes;
constexpr int kNq = kBN / kSplit;                 // 32 output columns summed by each rank
constexpr int kRecvPitch = kNq + 4;               // floats per row of a received block (16-byte aligned,
                                                  // 8 consecutive rows in distinct bank groups)
constexpr int kRecvBytes = kSplit * kBM * kRecvPitch * 4;  // [source rank][row][kRecvPitch] fp32
constexpr int kThreads = 128;
constexpr int kTmemCols = 256;
static_assert(kRecvBytes <= kStages * kStageBytes, "the receive blocks reuse the stage ring");
static_assert(kChunks >= kStages, "the producer requests the first kStages weight chunks up front");
constexpr uint32_t kIdesc = idesc_bf16_f32(128, kBN, 0, 0);

struct Smem {
    uint64_t full[kStages], empty[kStages];
    uint64_t done, ready, recv;
    uint32_t ready_word[kSplit];
    uint32_t tmem;
    int abort;
};
constexpr int kSmemBytes = kStages * kStageBytes + (int)sizeof(Smem) + 1024;
static_assert(kSmemBytes <= 232448, "K0 (tcgen05) shared memory exceeds 227 KB");
}  // namespace k0w

template <int kEpi>  // 0: bf16(sum), 1: bf16(residual + bf16(sum))
__global__ void __launch_bounds__(k0w::kThreads, 1)
    k_project_tc(const GemmArgs a, const __grid_constant__ CUtensorMap tmap_x,
                 const __grid_constant__ CUtensorMap tmap_w) {
    using namespace k0w;
    MLA_TL_SCOPE(4);
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    Smem& S = *reinterpret_cast<Smem*>(smem + kStages * kStageBytes);
    float* recv = reinterpret_cast<float*>(smem);  // after every rank's MMAs: [source][row][kRecvPitch]
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int rank = (int)cluster_rank();            // the K quarter of this CTA
    const int n0 = (blockIdx.x / kSplit) * kBN;
    const int m0 = blockIdx.y * kBM;
    const int mt = min(2, (a.batch - m0 + 127) / 128);  // M tiles that hold batch rows
    volatile int* abort = &S.abort;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; ++s) { mbar_init(&S.full[s], 1); mbar_init(&S.empty[s], 1); }
        mbar_init(&S.done, 1);
        mbar_init(&S.ready, 1);
        mbar_init(&S.recv, 1);
        S.abort = 0;
        fence_mbar_init();
        // bytes the peers will complete here: a 4-byte "ready" from each, then 128 B per
        // row of each M tile from each
        mbar_arrive_expect_tx(&S.ready, (kSplit - 1) * 4);
        mbar_arrive_expect_tx(&S.recv, (uint32_t)(kSplit - 1) * mt * 128 * kNq * 4);
        prefetch_tmap(&tmap_x);
        prefetch_tmap(&tmap_w);
    }
    if (warp == 1) {
        tmem_alloc(&S.tmem, kTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    cluster_sync_all();  // every rank's barriers are initialised before any peer completes bytes on them
    const uint32_t tmem = S.tmem;
    const int k_blk0 = rank * kChunks;  // first 64-column block of this quarter

    if (warp == 0 && lane == 0) {  // the weight's first chunks: no kernel writes it
        for (int c = 0; c < kStages; ++c) {
            mbar_arrive_expect_tx(&S.full[c], kStageBytes);
            tma_load_3d(smem + c * kStageBytes + kABytes, &tmap_w, &S.full[c], 0, n0, k_blk0 + c, kCacheEvictFirst);
        }
    }
    pdl_wait();  // x (and the residual) come from earlier work on the stream
    MLA_TL_WAITED(4);
    pdl_trigger();

    if (warp == 0) {
        // ------------------------------------------------------------ producer
        if (lane == 0) {
            int c = 0;
            for (; c < kChunks; ++c) {
                const int s = c % kStages, n = c / kStages;
                if (n > 0) {
                    if (!mbar_wait(&S.empty[s], (n - 1) & 1, abort, a.err)) break;
                    mbar_arrive_expect_tx(&S.full[s], kStageBytes);
                    tma_load_3d(smem + s * kStageBytes + kABytes, &tmap_w, &S.full[s], 0, n0, k_blk0 + c,
                                kCacheEvictFirst);
                }
                tma_load_3d(smem + s * kStageBytes, &tmap_x, &S.full[s], 0, m0, k_blk0 + c, kCacheEvictLast);
            }
            // Drain: every issued copy lands before the ring is reused or released (the
            // loop issues both copies of the first kStages chunks without a wait, so c >= kStages)
            for (int s = 0; s < kStages; ++s) {
                const int fills = c / kStages + (s < c % kStages ? 1 : 0);
                if (fills) mbar_drain(&S.full[s], (fills - 1) & 1, a.err);
            }
        }
    } else if (warp == 1) {
        // ------------------------------------------------------------ MMA issuer
        if (lane == 0) {
            const uint32_t base = smem_u32(smem);
            const uint64_t dK = smem_desc_sw128(0, 16, 1024);  // K-major, 8-row groups 1024 B apart
            for (int c = 0; c < kChunks; ++c) {
                const int s = c % kStages;
                if (!mbar_wait(&S.full[s], (c / kStages) & 1, abort, a.err)) break;
                tc_fence_after();
                const uint32_t sa = base + s * kStageBytes, sb = sa + kABytes;
#pragma unroll
                for (int kk = 0; kk < kKc / 16; ++kk) {
                    const uint64_t bd = dK + ((sb + kk * 32) >> 4);
                    for (int m = 0; m < mt; ++m) {
                        const uint64_t ad = dK + ((sa + m * (128 * 128) + kk * 32) >> 4);
                        tc_mma_f16(tmem + m * kBN, ad, bd, kIdesc, (c | kk) ? 1u : 0u);
                    }
                }
                tc_commit(&S.empty[s]);
            }
            tc_commit(&S.done);  // also after an abort: every issued MMA completes before the epilogue
        }
    }
    __syncwarp();

    // ---------------------------------------------------------------- epilogue (all warps)
    mbar_wait(&S.done, 0, abort, a.err);
    tc_fence_after();
    // this rank's stage ring is free: tell every peer, then wait until every peer's is
    if (threadIdx.x == 0) {
        const uint32_t wl = smem_u32(&S.ready_word[rank]), bl = smem_u32(&S.ready);
        for (int q = 0; q < kSplit; ++q)
            if (q != rank) dsmem_push1(dsmem_addr(wl, (uint32_t)q), 1u, dsmem_addr(bl, (uint32_t)q));
    }
    mbar_wait(&S.ready, 0, abort, a.err);
    // rows 32 warp + lane of each M tile: columns [32 q, 32 q + 32) go to rank q
    const uint32_t recv_l = smem_u32(recv), recv_bar = smem_u32(&S.recv);
    for (int m = 0; m < mt; ++m) {
        const int row = m * 128 + 32 * warp + lane;
#pragma unroll 1
        for (int q = 0; q < kSplit; ++q) {
            float v[32];
            const uint32_t ta = tmem_lane_addr(tmem, warp, m * kBN + kNq * q);
            tmem_ld16(ta, *reinterpret_cast<float(*)[16]>(v));
            tmem_ld16(ta + 16, *reinterpret_cast<float(*)[16]>(v + 16));
            tmem_wait_ld();
            const uint32_t off = (uint32_t)((rank * kBM + row) * kRecvPitch) * 4u;  // slot [rank][row] at q
            if (q == rank) {
#pragma unroll
                for (int j = 0; j < kNq; j += 4)
                    *reinterpret_cast<float4*>(recv + (rank * kBM + row) * kRecvPitch + j) =
                        make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
            } else {
                const uint32_t dst = dsmem_addr(recv_l + off, (uint32_t)q), bar = dsmem_addr(recv_bar, (uint32_t)q);
#pragma unroll
                for (int j = 0; j < kNq; j += 4)
                    dsmem_push4(dst + 4u * j, make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]), bar);
            }
        }
    }
    mbar_wait(&S.recv, 0, abort, a.err);
    tc_fence_before();
    __syncthreads();  // own block written; every tcgen05.ld done before the tensor memory is freed
    if (warp == 1) tmem_dealloc(tmem, kTmemCols);

    // sum of the four K quarters in rank order, epilogue, store (thread = one row of a tile)
    const int ncol0 = n0 + kNq * rank;
    for (int m = 0; m < mt; ++m) {
        const int row = m * 128 + threadIdx.x, b = m0 + row;
        if (b >= a.batch || ncol0 >= a.n_rows) continue;
        float acc[kNq];
#pragma unroll
        for (int j = 0; j < kNq; ++j) acc[j] = 0.f;
#pragma unroll
        for (int src = 0; src < kSplit; ++src) {
            const float* r = recv + (src * kBM + row) * kRecvPitch;
#pragma unroll
            for (int j = 0; j < kNq; j += 4) {
                const float4 x = *reinterpret_cast<const float4*>(r + j);
                acc[j] += x.x; acc[j + 1] += x.y; acc[j + 2] += x.z; acc[j + 3] += x.w;
            }
        }
        // 8-byte accesses: K5's residual and h_out rows are 8-byte aligned (strides of 4 elements)
        __nv_bfloat16* yrow = a.y + (int64_t)b * a.y_stride + ncol0;
        const __nv_bfloat16* rrow = kEpi ? a.residual + (int64_t)b * a.res_stride + ncol0 : nullptr;
#pragma unroll
        for (int j = 0; j < kNq; j += 4) {
            if (ncol0 + j >= a.n_rows) break;  // the last tile of K0's 3648 rows is half full
            float v[4] = {acc[j], acc[j + 1], acc[j + 2], acc[j + 3]};
            if (kEpi) {
                const uint2 rv = *reinterpret_cast<const uint2*>(rrow + j);
                const __nv_bfloat162* r2 = reinterpret_cast<const __nv_bfloat162*>(&rv);
                v[0] = __low2float(r2[0]) + bf16_round(v[0]);
                v[1] = __high2float(r2[0]) + bf16_round(v[1]);
                v[2] = __low2float(r2[1]) + bf16_round(v[2]);
                v[3] = __high2float(r2[1]) + bf16_round(v[3]);
            }
            uint2 o;
            o.x = pack_bf16(v[0], v[1]);
            o.y = pack_bf16(v[2], v[3]);
            *reinterpret_cast<uint2*>(yrow + j) = o;
        }
    }
}

cudaError_t k0w_configure() {
    cudaError_t e = cudaFuncSetAttribute(k_project_tc<0>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         k0w::kSmemBytes);
    if (e != cudaSuccess) return e;
    return cudaFuncSetAttribute(k_project_tc<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, k0w::kSmemBytes);
}

// x [batch][2048] (row pitch x_stride elements) and W [n_rows][2048] as the operand maps
// of the kernel: dims {64 columns, rows, 32 column blocks}, 128-byte swizzle, boxes of
// 256 (x) and 128 (W) rows by one 64-column block.
cudaError_t launch_project_tc(int epi, const GemmArgs& a, const CUtensorMap& tmap_x, const CUtensorMap& tmap_w,
                              cudaStream_t stream) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(((a.n_rows + k0w::kBN - 1) / k0w::kBN) * k0w::kSplit, (a.batch + k0w::kBM - 1) / k0w::kBM);
    cfg.blockDim = dim3(k0w::kThreads);
    cfg.dynamicSmemBytes = k0w::kSmemBytes;
    cfg.stream = stream;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = k0w::kSplit;
    attr[1].val.clusterDim.y = 1;
    attr[1].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    return epi ? cudaLaunchKernelEx(&cfg, k_project_tc<1>, a, tmap_x, tmap_w)
               : cudaLaunchKernelEx(&cfg, k_project_tc<0>, a, tmap_x, tmap_w);
}

}  // namespace mla
