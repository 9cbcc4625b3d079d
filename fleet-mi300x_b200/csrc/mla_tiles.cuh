// Split-KV tile walking and warp helpers shared by the attention kernels.
#pragma once

#include "mla_common.cuh"

namespace mla {

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
    int extra;  // 1 if the new token's row is part of the attended rows

    __device__ void init(const int32_t* cum_, const int32_t* sl, int B, int64_t ub, int64_t ue, int extra_ = 1) {
        cum = cum_; seq_lens = sl; batch = B; u = ub; u_begin = ub; u_end = ue; seg = 0; extra = extra_;
        // largest b with cum[b] <= u (upper_bound - 1); skips empty requests
        int lo = 0, hi = B;  // cum[B] > u
        while (hi - lo > 1) {
            const int mid = (lo + hi) >> 1;
            if (cum[mid] <= u) lo = mid; else hi = mid;
        }
        b = lo; cb0 = cum[b]; cb1 = cum[b + 1];
    }
    // The same start from a plan entry (no search).
    __device__ void init_at(const int32_t* cum_, const int32_t* sl, int B, const PlanEntry& e, int extra_ = 1) {
        cum = cum_; seq_lens = sl; batch = B; u = e.u_begin; u_begin = e.u_begin; u_end = e.u_end; seg = 0;
        extra = extra_;
        b = e.b; cb0 = e.cb0; cb1 = e.cb1;
    }
    __device__ bool valid() const { return u < u_end; }
    __device__ int index() const { return (int)(u - cb0); }       // tile of the current request
    __device__ int page_index() const { return (int)(u - cb0); }  // the same, for 64-row tiles
    __device__ int tokens() const {  // valid tokens in this 64-token tile
        const int L = seq_lens[b] + extra;
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
__device__ __forceinline__ void mbar_drain(uint64_t* bar, uint32_t parity, const ErrSink& err) {
    int dummy = 0;
    mbar_wait(bar, parity, &dummy, err);
}

}  // namespace mla
