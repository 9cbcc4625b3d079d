// The two projections around the attention task for batches beyond the weight
// stream's 64 requests, on the 5th-generation tensor cores:
//   K0: q | kv_a = R(x_n [W_q; W_kv_a]^T)             (reference_decode.py:225-231)
//   K5: h' = R(h + R(R(out) W_o^T))                    (reference_decode.py:256, 300)
// y[b][n] = epi(sum_k x[b][k] W[n][k]) over K = 2048, for N = 3648 (K0) or 2048
// (K5) weight rows. At 64 requests or fewer the weight is the whole cost and the
// weight-stream kernel (mla_project.cu) runs instead; beyond that the product is
// a GEMM (3.8 GFLOP at 256 requests for K0) with M = batch.
//
// Tiling: a CTA owns 128 batch rows (one M = 128 tcgen05 tile) x 64 weight rows
// (N = 64) over the whole K, so no partial sums cross CTAs and the epilogue goes
// from tensor memory straight to global memory (K0 at 256 requests: 57 x 2 = 114
// CTAs). Warp roles:
//   * warp 0, one thread: TMA producer. Per 256-column chunk of K (8 chunks), one
//     box of x (128 rows x 4 column blocks, 64 KB; rows past the batch read as
//     zeros) and one of W (64 rows x 4 blocks, 32 KB; rows past N as zeros) into a
//     2-stage ring (192 KB in flight). Large boxes: a copy engine moves far more
//     bytes per SM in few large requests than in many 8-16 KB ones. The first two W
//     chunks are requested before the wait on the previous kernel (no kernel
//     writes a weight). No multicast.
//   * warp 1: allocates 64 columns of tensor memory (D, fp32) and one thread
//     issues tcgen05.mma (kind::f16, bf16 operands, both K-major in 128-byte
//     swizzled tiles), 16 K-steps per chunk, committing each stage back to the
//     producer and the last one to the epilogue.
//   * all 4 warps, epilogue: warp w reads its 32 lanes (batch rows) of D, rounds
//     (K5: adds the residual and rounds again) and stores 64 bf16 per row.
// Every wait is bounded (mla::mbar_wait); a timeout is recorded in the error word.
//
// Measured at 256 requests, L2 flushed before each call (1x B200): 17.4 us, against
// 12.9 us for cuBLAS's GEMM on the same operands. Each of the 114 CTAs streams 768 KB
// (its 128 rows of x and 64 rows of W over all of K) at about 50 GB/s. cuBLAS's kernel
// here is a 2 x 4-cluster kernel by its name, whose CTAs can share operand tiles
// within a cluster; this library uses no cluster multicast loads (its code also runs
// on several GPUs), so the Python host keeps cuBLAS above 64 requests and this kernel serves C
// callers (the x_n / w_o fields) that want the whole block without cuBLAS. Measured
// and not kept: 24 KB stages (20.5 us), 48 KB stages (18.4 us), and K split over a
// 4-CTA cluster with the partials summed through distributed shared memory (21.8 us:
// 96 KB of 16-byte pushes per CTA).
#include <cuda.h>

#include "mla_common.cuh"
#include "mla_mma.cuh"
#include "mla_tiles.cuh"

namespace mla {

namespace k0w {
constexpr int kBM = 128;                          // batch rows per CTA: the MMA's M
constexpr int kBN = 64;                           // weight rows per CTA: the MMA's N
constexpr int kBlk = 4;                           // 64-column blocks (128-byte swizzle atoms) per chunk
constexpr int kKc = 64 * kBlk;                    // K per chunk: 256
constexpr int kChunks = kHidden / kKc;            // 8
constexpr int kStages = 2;
constexpr int kABlock = kBM * 128;                // 16384: one block of x, [128 rows][128 B]
constexpr int kBBlock = kBN * 128;                // 8192: one block of W, [64 rows][128 B]
constexpr int kABytes = kBlk * kABlock;           // 65536
constexpr int kBBytes = kBlk * kBBlock;           // 32768
constexpr int kStageBytes = kABytes + kBBytes;    // 96 KB, a multiple of 1024 (swizzle atoms stay aligned)
constexpr int kThreads = 128;
constexpr int kTmemCols = 64;
static_assert(kChunks >= kStages, "the producer requests the first kStages weight chunks up front");
static_assert(kStageBytes % 1024 == 0, "stages must stay 1024-byte aligned");
constexpr uint32_t kIdesc = idesc_bf16_f32(kBM, kBN, 0, 0);

struct Smem {
    uint64_t full[kStages], empty[kStages];
    uint64_t done;
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
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n0 = blockIdx.x * kBN;
    const int m0 = blockIdx.y * kBM;
    // K order rotated per weight tile: the tiles of one batch block read different
    // chunks of x at any moment instead of all the same L2 lines at once
    const int k_rot = blockIdx.x % kChunks;
    volatile int* abort = &S.abort;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; ++s) { mbar_init(&S.full[s], 1); mbar_init(&S.empty[s], 1); }
        mbar_init(&S.done, 1);
        S.abort = 0;
        fence_mbar_init();
        prefetch_tmap(&tmap_x);
        prefetch_tmap(&tmap_w);
        for (int c = 0; c < kStages; ++c) {  // the weight's first chunks: no kernel writes it
            mbar_arrive_expect_tx(&S.full[c], kStageBytes);
            tma_load_3d(smem + c * kStageBytes + kABytes, &tmap_w, &S.full[c], 0, n0,
                        kBlk * ((c + k_rot) % kChunks), kCacheEvictFirst);
        }
    }
    if (warp == 1) {
        tmem_alloc(&S.tmem, kTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = S.tmem;
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
                    tma_load_3d(smem + s * kStageBytes + kABytes, &tmap_w, &S.full[s], 0, n0,
                                kBlk * ((c + k_rot) % kChunks), kCacheEvictFirst);
                }
                tma_load_3d(smem + s * kStageBytes, &tmap_x, &S.full[s], 0, m0, kBlk * ((c + k_rot) % kChunks),
                            kCacheEvictLast);
            }
            // Drain: every issued copy lands before the ring is released (both copies of
            // the first kStages chunks go out without a wait, so c >= kStages here).
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
                for (int j = 0; j < kBlk; ++j)
#pragma unroll
                    for (int kk = 0; kk < 4; ++kk)
                        tc_mma_f16(tmem, dK + ((sa + j * kABlock + kk * 32) >> 4),
                                   dK + ((sb + j * kBBlock + kk * 32) >> 4), kIdesc, (c | j | kk) ? 1u : 0u);
                tc_commit(&S.empty[s]);
            }
            tc_commit(&S.done);  // also after an abort: every issued MMA completes before the epilogue
        }
    }
    __syncwarp();

    // ---------------------------------------------------------------- epilogue (all warps)
    mbar_wait(&S.done, 0, abort, a.err);
    tc_fence_after();
    const int row = 32 * warp + lane, b = m0 + row;
    float v[kBN];
#pragma unroll
    for (int j = 0; j < kBN; j += 16)
        tmem_ld16(tmem_lane_addr(tmem, warp, j), *reinterpret_cast<float(*)[16]>(v + j));
    tmem_wait_ld();
    tc_fence_before();
    __syncthreads();  // every tcgen05.ld done before the tensor memory is freed
    if (warp == 1) tmem_dealloc(tmem, kTmemCols);
    if (b >= a.batch) return;
    // 8-byte accesses: K5's residual and h_out rows are 8-byte aligned (strides of 4 elements)
    __nv_bfloat16* yrow = a.y + (int64_t)b * a.y_stride + n0;
    const __nv_bfloat16* rrow = kEpi ? a.residual + (int64_t)b * a.res_stride + n0 : nullptr;
#pragma unroll
    for (int j = 0; j < kBN; j += 4) {
        if (n0 + j >= a.n_rows) break;  // the last tile of K0's 3648 rows is half full
        float o[4] = {v[j], v[j + 1], v[j + 2], v[j + 3]};
        if (kEpi) {
            const uint2 rv = *reinterpret_cast<const uint2*>(rrow + j);
            const __nv_bfloat162* r2 = reinterpret_cast<const __nv_bfloat162*>(&rv);
            o[0] = __low2float(r2[0]) + bf16_round(o[0]);
            o[1] = __high2float(r2[0]) + bf16_round(o[1]);
            o[2] = __low2float(r2[1]) + bf16_round(o[2]);
            o[3] = __high2float(r2[1]) + bf16_round(o[3]);
        }
        uint2 st;
        st.x = pack_bf16(o[0], o[1]);
        st.y = pack_bf16(o[2], o[3]);
        *reinterpret_cast<uint2*>(yrow + j) = st;
    }
}

cudaError_t k0w_configure() {
    cudaError_t e = cudaFuncSetAttribute(k_project_tc<0>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         k0w::kSmemBytes);
    if (e != cudaSuccess) return e;
    return cudaFuncSetAttribute(k_project_tc<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, k0w::kSmemBytes);
}

int k0w_box_rows_x() { return k0w::kBM; }
int k0w_box_rows_w() { return k0w::kBN; }
int k0w_box_blocks() { return k0w::kBlk; }

// x [batch][2048] (row pitch x_stride elements) and W [n_rows][2048] as the operand maps
// of the kernel: dims {64 columns, rows, 32 column blocks}, 128-byte swizzle, boxes of
// k0w_box_rows_x() / k0w_box_rows_w() rows by k0w_box_blocks() 64-column blocks.
cudaError_t launch_project_tc(int epi, const GemmArgs& a, const CUtensorMap& tmap_x, const CUtensorMap& tmap_w,
                              cudaStream_t stream) {
    const dim3 grid((a.n_rows + k0w::kBN - 1) / k0w::kBN, (a.batch + k0w::kBM - 1) / k0w::kBM);
    return epi ? launch_pdl(k_project_tc<1>, grid, dim3(k0w::kThreads), k0w::kSmemBytes, stream, a, tmap_x, tmap_w)
               : launch_pdl(k_project_tc<0>, grid, dim3(k0w::kThreads), k0w::kSmemBytes, stream, a, tmap_x, tmap_w);
}

}  // namespace mla
