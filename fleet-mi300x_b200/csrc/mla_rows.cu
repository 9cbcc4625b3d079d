// Prefill hand-off: rows of a prefill into the paged latent cache.
//
// The reference hands prefill states to decode as one flat cache per layer,
// [max_pos][576] bf16 rows c (after kv_a_layernorm) | k_pe (after RoPE), built
// from the hooked kv_a_proj_with_mqa output (src/host/kv_convert.py:36-139)
// and uploaded by the launcher as-is (src/host/fleet_launch.hip:651-669). Here
// the cache is paged, so the hand-off scatters each request's rows into its
// pages: MLA_ROWS_FINAL copies finished rows (the reference's file format);
// MLA_ROWS_RAW takes raw kv_a rows and applies kv_a_layernorm and RoPE at each
// row's position with the same arithmetic as the decode step's appended row.
//
// One warp per row, 8 rows per CTA, grid-stride. Bounds are checked per row:
// a position outside the block table (or, for raw rows, outside the RoPE
// tables) records MLA_DEV_BAD_POSITION and a page id outside the pool records
// MLA_DEV_BAD_PAGE; such rows are skipped. HBM-bound: 1,152 B read and 1,152 B
// written per row.
#include "mla_common.cuh"
#include "mla_rowops.cuh"

namespace mla {

constexpr int kRowsThreads = 256;
constexpr int kRowsPerCta = kRowsThreads / 32;

__global__ void __launch_bounds__(kRowsThreads) k_rows_to_pages(const MlaRowsToPages r) {
    const int lane = threadIdx.x & 31;
    const __nv_bfloat16* rows = reinterpret_cast<const __nv_bfloat16*>(r.rows);
    __nv_bfloat16* cache = reinterpret_cast<__nv_bfloat16*>(r.kv_cache);
    for (int64_t i = (int64_t)blockIdx.x * kRowsPerCta + (threadIdx.x >> 5); i < r.total_rows;
         i += (int64_t)gridDim.x * kRowsPerCta) {
        // request of row i: largest b with row_start[b] <= i
        int lo = 0, hi = r.batch;
        while (hi - lo > 1) {
            const int mid = (lo + hi) >> 1;
            if (r.row_start[mid] <= i) lo = mid; else hi = mid;
        }
        const int b = lo;
        const int64_t pos64 = (r.first_pos ? r.first_pos[b] : 0) + (i - r.row_start[b]);
        const bool raw = r.mode == MLA_ROWS_RAW;
        if (pos64 < 0 || pos64 >= (int64_t)r.max_blocks * kPage || (raw && pos64 >= r.max_pos)) {
            if (lane == 0) record_error(ErrSink{r.error_word, nullptr}, MLA_DEV_BAD_POSITION);
            continue;
        }
        const int pos = (int)pos64;
        const int page = r.block_table[(int64_t)b * r.max_blocks + pos / kPage];
        if (page < 0 || page >= r.n_pages) {
            if (lane == 0) record_error(ErrSink{r.error_word, nullptr}, MLA_DEV_BAD_PAGE);
            continue;
        }
        const __nv_bfloat16* src = rows + i * r.rows_stride;
        __nv_bfloat16* dst = cache + ((int64_t)page * kPage + pos % kPage) * kRow;
        if (raw) {
            __align__(16) __nv_bfloat16 outc[16];
            float rlo, rhi;
            kv_post_compute(src, reinterpret_cast<const __nv_bfloat16*>(r.kv_a_norm_w), r.rms_eps,
                            r.rope_cos + (int64_t)pos * kRope, r.rope_sin + (int64_t)pos * kRope, lane, outc, rlo,
                            rhi);
            kv_post_store(dst, outc, rlo, rhi, lane);
        } else {
            const uint4* s4 = reinterpret_cast<const uint4*>(src);
            uint4* d4 = reinterpret_cast<uint4*>(dst);
            const uint4 a = s4[lane], c = s4[lane + 32];
            uint4 e = make_uint4(0u, 0u, 0u, 0u);
            if (lane < kRow / 8 - 64) e = s4[lane + 64];
            d4[lane] = a;
            d4[lane + 32] = c;
            if (lane < kRow / 8 - 64) d4[lane + 64] = e;
        }
    }
}

cudaError_t launch_rows_to_pages(const MlaRowsToPages& r, int sm_count, cudaStream_t stream) {
    const int64_t need = (r.total_rows + kRowsPerCta - 1) / kRowsPerCta;
    const int64_t cap = (int64_t)sm_count * 16;
    const int grid = (int)(need < cap ? need : cap);
    if (grid <= 0) return cudaSuccess;
    k_rows_to_pages<<<grid, kRowsThreads, 0, stream>>>(r);
    return cudaGetLastError();
}

}  // namespace mla
