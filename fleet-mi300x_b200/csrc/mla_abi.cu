// extern "C" entry points of libmla_decode.so (declared in include/mla_decode.h).
//
// Host glue that replaces the attention part of the reference's launcher
// (src/host/fleet_launch.hip): the shape refusal (:573-577), the per-launch
// argument packing and launch (fleet_kernel.hip:1068-1078) and the error
// decoding (:284-311). The YaRN tables and softmax scale (:186-219, :564-571)
// are computed by the caller (the Python host) and passed in.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <cstring>
#include <mutex>

#include "mla_common.cuh"

namespace mla {
cudaError_t launch_prologue(const MlaDecodeParams& p, const CUtensorMap& tmap_kvb, cudaStream_t stream);
cudaError_t launch_attention_tc(const MlaDecodeParams& p, const CUtensorMap& tmap_kv, const CUtensorMap& tmap_q,
                                float scale_log2, cudaStream_t stream);
cudaError_t launch_attention_check(const MlaDecodeParams& p, float scale_log2, cudaStream_t stream);
cudaError_t launch_merge_uv(const MlaDecodeParams& p, const CUtensorMap& tmap_kvb, int sm_count, bool fused,
                            cudaStream_t stream);
bool k3_fused_fits(int batch, int sm_count);
cudaError_t k1_configure();
cudaError_t launch_combine_shards(const float* parts, int n_shards, int batch, void* out, int64_t out_stride,
                                  cudaStream_t stream);
cudaError_t launch_exchange_combine(const MlaDecodeParams& p, cudaStream_t stream);
cudaError_t launch_attention_mma(const MlaDecodeParams& p, const CUtensorMap& tmap_kv, float scale_log2,
                                 int sm_count, cudaStream_t stream);
cudaError_t k2_configure();
cudaError_t k2_mma_configure();
cudaError_t k3_configure();
int k3_w_rows(int batch);
cudaError_t k0_configure();
cudaError_t launch_rows_to_pages(const MlaRowsToPages& r, int sm_count, cudaStream_t stream);
cudaError_t launch_o_proj(const MlaDecodeParams& p, const CUtensorMap& tmap_w, const CUtensorMap& tmap_x,
                          cudaStream_t stream);
cudaError_t launch_project(const MlaDecodeParams& p, __nv_bfloat16* qkv, const CUtensorMap& tmap_w,
                           const CUtensorMap& tmap_x, cudaStream_t stream);
cudaError_t k0w_configure();
int k0w_box_rows_x();
int k0w_box_rows_w();
int k0w_box_blocks();
cudaError_t launch_project_tc(int epi, const GemmArgs& a, const CUtensorMap& tmap_x, const CUtensorMap& tmap_w,
                              cudaStream_t stream);

namespace {

constexpr int kMaxDevices = 64;
constexpr int kMaxCtas = 4096;

struct DeviceInfo {
    std::once_flag once;
    int status = MLA_E_ARCH;
    int sm_count = 0;
};
DeviceInfo g_dev[kMaxDevices];

PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
std::once_flag g_encode_once;

int device_info(int* sm_count) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return MLA_E_LAUNCH;
    DeviceInfo& d = g_dev[dev];
    std::call_once(d.once, [&]() {
        cudaDeviceProp prop;
        if (cudaGetDeviceProperties(&prop, dev) != cudaSuccess) { d.status = MLA_E_LAUNCH; return; }
        if (prop.major != 10) { d.status = MLA_E_ARCH; return; }
        if (k0_configure() != cudaSuccess || k0w_configure() != cudaSuccess || k1_configure() != cudaSuccess ||
            k2_configure() != cudaSuccess || k2_mma_configure() != cudaSuccess || k3_configure() != cudaSuccess) {
            d.status = MLA_E_LAUNCH;
            return;
        }
        d.sm_count = prop.multiProcessorCount;
        d.status = MLA_OK;
    });
    if (d.status == MLA_OK && sm_count) *sm_count = d.sm_count;
    return d.status;
}

int encode_fn(PFN_cuTensorMapEncodeTiled_v12000* fn) {
    std::call_once(g_encode_once, []() {
        void* f = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &f, 12000, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(f);
    });
    *fn = g_encode;
    return g_encode ? MLA_OK : MLA_E_DRIVER;
}

// bf16 tensor maps over 576-wide rows (1152 B pitch) that land in shared
// memory as 9 column blocks of [rows x 64] with the 128-byte swizzle:
// dims {64 columns, rows (pitch 1152 B), 9 blocks (pitch 128 B)[, pages]}.
// The page map (rank 4) serves box_rows rows of one page per request (64: a
// whole page, the tcgen05 kernel; 32: half a page, the m16n8k16 kernel); the
// query map (rank 3) one request's 16 absorbed-query rows.
int make_tmap_blocks(CUtensorMap* m, const void* base, uint64_t rows_or_pages, bool paged, int box_rows) {
    PFN_cuTensorMapEncodeTiled_v12000 fn;
    if (encode_fn(&fn) != MLA_OK) return MLA_E_DRIVER;
    const cuuint32_t rank = paged ? 4 : 3;
    cuuint64_t dims[4] = {64, paged ? (cuuint64_t)kPage : (cuuint64_t)rows_or_pages, 9, (cuuint64_t)rows_or_pages};
    cuuint64_t strides[3] = {(cuuint64_t)kRow * 2, 128, (cuuint64_t)kPage * kRow * 2};
    cuuint32_t box[4] = {64, (cuuint32_t)box_rows, 9, 1};
    cuuint32_t estr[4] = {1, 1, 1, 1};
    CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, rank, const_cast<void*>(base), dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_NONE,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? MLA_OK : MLA_E_DRIVER;
}

// kv_b (16*256 rows x 512 bf16) as row blocks of W_UK / W_UV: dims {64 columns,
// 4096 rows (1024 B), 8 column blocks (128 B)}, box {64, box_rows, blocks} = one
// request of box_rows x blocks x 128 B landing as [blocks][box_rows rows][128 B]
// with the 128-byte swizzle (128 x 8: a whole 128 x 512 head block for the plain
// merge; 32 x 8: a cluster CTA's rows of W_UV; 128 x 2: a quarter of W_UK's columns).
int make_tmap_kvb(CUtensorMap* m, const void* kv_b, int box_rows, int blocks) {
    PFN_cuTensorMapEncodeTiled_v12000 fn;
    if (encode_fn(&fn) != MLA_OK) return MLA_E_DRIVER;
    cuuint64_t dims[3] = {64, (cuuint64_t)kHeads * kKvbHead, 8};
    cuuint64_t strides[2] = {(cuuint64_t)kLora * 2, 128};
    cuuint32_t box[3] = {64, (cuuint32_t)box_rows, (cuuint32_t)blocks};
    cuuint32_t estr[3] = {1, 1, 1};
    CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(kv_b), dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_NONE,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? MLA_OK : MLA_E_DRIVER;
}

// A [rows x 2048] bf16 weight (the stacked [W_q; W_kv_a], 3648 rows, or W_o,
// 2048 rows) as dims {64 columns, rows (4096 B), 32 column blocks (128 B)}, box
// {64, box_rows, 8}: box_rows weight rows x 512 columns landing as
// [8][box_rows rows][128 B] (128-byte swizzle).
int make_tmap_weight(CUtensorMap* m, const void* w, int rows, int box_rows) {
    PFN_cuTensorMapEncodeTiled_v12000 fn;
    if (encode_fn(&fn) != MLA_OK) return MLA_E_DRIVER;
    cuuint64_t dims[3] = {64, (cuuint64_t)rows, kHidden / 64};
    cuuint64_t strides[2] = {(cuuint64_t)kHidden * 2, 128};
    cuuint32_t box[3] = {64, (cuuint32_t)box_rows, 8};
    cuuint32_t estr[3] = {1, 1, 1};
    CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(w), dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_NONE,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? MLA_OK : MLA_E_DRIVER;
}

// x_n (batch rows x 2048 bf16, row pitch x_stride) as dims {64 columns, batch
// rows, 32 column blocks}, box {64, 16, 32}: 16 rows x 2048 = 64 KB landing as
// [32][16 rows][128 B]; rows past the batch read as zeros.
int make_tmap_x(CUtensorMap* m, const void* x, int batch, int64_t x_stride) {
    PFN_cuTensorMapEncodeTiled_v12000 fn;
    if (encode_fn(&fn) != MLA_OK) return MLA_E_DRIVER;
    cuuint64_t dims[3] = {64, (cuuint64_t)batch, kHidden / 64};
    cuuint64_t strides[2] = {(cuuint64_t)x_stride * 2, 128};
    cuuint32_t box[3] = {64, 16, kHidden / 64};
    cuuint32_t estr[3] = {1, 1, 1};
    CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(x), dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_NONE,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? MLA_OK : MLA_E_DRIVER;
}

// [rows][2048] bf16 with a row pitch of `stride` elements as an operand of the
// tensor-core projection: dims {64 columns, rows, 32 column blocks}, box {64,
// box_rows, blocks} (landing as [blocks][box_rows rows][128 B], 128-byte swizzle);
// rows past `rows` read as zeros.
int make_tmap_operand(CUtensorMap* m, const void* base, int rows, int64_t stride, int box_rows, int blocks) {
    PFN_cuTensorMapEncodeTiled_v12000 fn;
    if (encode_fn(&fn) != MLA_OK) return MLA_E_DRIVER;
    cuuint64_t dims[3] = {64, (cuuint64_t)rows, kHidden / 64};
    cuuint64_t strides[2] = {(cuuint64_t)stride * 2, 128};
    cuuint32_t box[3] = {64, (cuuint32_t)box_rows, (cuuint32_t)blocks};
    cuuint32_t estr[3] = {1, 1, 1};
    CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_NONE,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? MLA_OK : MLA_E_DRIVER;
}

// Batches beyond MLA_MAX_PROJECT_BATCH: the projection as a tensor-core GEMM (epi 0:
// y = bf16(x W^T); epi 1: y = bf16(residual + bf16(x W^T))).
int run_gemm_tc(int epi, const GemmArgs& a, const void* x, int64_t x_stride, const void* w, cudaStream_t s) {
    CUtensorMap tx, tw;
    int st = make_tmap_operand(&tx, x, a.batch, x_stride, k0w_box_rows_x(), k0w_box_blocks());
    if (st != MLA_OK) return st;
    st = make_tmap_operand(&tw, w, a.n_rows, kHidden, k0w_box_rows_w(), k0w_box_blocks());
    if (st != MLA_OK) return st;
    return launch_project_tc(epi, a, tx, tw, s) == cudaSuccess ? MLA_OK : MLA_E_LAUNCH;
}

int run_project(const MlaDecodeParams& q, cudaStream_t s) {
    if (q.batch > MLA_MAX_PROJECT_BATCH) {
        __nv_bfloat16* qkv =
            reinterpret_cast<__nv_bfloat16*>(reinterpret_cast<char*>(q.workspace) + ws_layout(q).qkv);
        const GemmArgs a{qkv, kQkvRows, nullptr, 0, q.batch, kQkvRows, err_sink(q)};
        return run_gemm_tc(0, a, q.x_n, q.x_stride, q.w_qkv, s);
    }
    CUtensorMap tw, tx;
    int st = make_tmap_weight(&tw, q.w_qkv, kQkvRows, 32);
    if (st != MLA_OK) return st;
    st = make_tmap_x(&tx, q.x_n, q.batch, q.x_stride);
    if (st != MLA_OK) return st;
    __nv_bfloat16* qkv = reinterpret_cast<__nv_bfloat16*>(reinterpret_cast<char*>(q.workspace) + ws_layout(q).qkv);
    return launch_project(q, qkv, tw, tx, s) == cudaSuccess ? MLA_OK : MLA_E_LAUNCH;
}

int run_o_proj(const MlaDecodeParams& q, cudaStream_t s) {
    if (q.batch > MLA_MAX_PROJECT_BATCH) {
        const GemmArgs a{reinterpret_cast<__nv_bfloat16*>(q.h_out), q.h_out_stride,
                         reinterpret_cast<const __nv_bfloat16*>(q.residual), q.residual_stride, q.batch, kHidden,
                         err_sink(q)};
        return run_gemm_tc(1, a, q.out, q.out_stride, q.w_o, s);
    }
    CUtensorMap tw, tx;
    int st = make_tmap_weight(&tw, q.w_o, kHidden, 16);
    if (st != MLA_OK) return st;
    st = make_tmap_x(&tx, q.out, q.batch, q.out_stride);
    if (st != MLA_OK) return st;
    return launch_o_proj(q, tw, tx, s) == cudaSuccess ? MLA_OK : MLA_E_LAUNCH;
}

int run_prologue(const MlaDecodeParams& q, cudaStream_t s) {
    CUtensorMap t;
    const int st = make_tmap_kvb(&t, q.kv_b, 128, kK1WukBlocks);
    if (st != MLA_OK) return st;
    return launch_prologue(q, t, s) == cudaSuccess ? MLA_OK : MLA_E_LAUNCH;
}

int run_merge(const MlaDecodeParams& q, cudaStream_t s, bool fused = false) {
    CUtensorMap t;
    int st = make_tmap_kvb(&t, q.kv_b, k3_w_rows(q.batch), 8);
    if (st != MLA_OK) return st;
    int sms = 0;
    st = device_info(&sms);
    if (st != MLA_OK) return st;
    return launch_merge_uv(q, t, sms, fused, s) == cudaSuccess ? MLA_OK : MLA_E_LAUNCH;
}

// Whether this step's peer exchange runs fused into K3 (no K4): the whole K3 grid
// must be resident at once. The answer depends only on the batch and the device;
// the last one is kept per device.
struct FusedCache {
    std::mutex mu;
    int batch = -1;
    bool fits = false;
};
FusedCache g_fused[kMaxDevices];

bool exchange_fused(const MlaDecodeParams& q) {
    if (q.world <= 0 || (q.flags & MLA_FLAG_EXCHANGE_SPLIT)) return false;
    int dev = 0, sms = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices || device_info(&sms) != MLA_OK)
        return false;
    FusedCache& c = g_fused[dev];
    std::lock_guard<std::mutex> lock(c.mu);
    if (c.batch != q.batch) {
        c.fits = k3_fused_fits(q.batch, sms);
        c.batch = q.batch;
    }
    return c.fits;
}

bool aligned(const void* ptr, uintptr_t a) { return (reinterpret_cast<uintptr_t>(ptr) & (a - 1)) == 0; }

// CTAs of the split plan: p->num_ctas, or by default as many as run at once:
// two per SM for the m16n8k16 kernel (each of its CTAs runs two plan CTAs as
// independent warp groups) and the checker, one per SM for the tcgen05 kernel.
int resolve_ctas(const MlaDecodeParams* p, int* ctas) {
    if (p->num_ctas < 0 || p->num_ctas > kMaxCtas) return MLA_E_LIMIT;
    if (p->num_ctas > 0) { *ctas = p->num_ctas; return MLA_OK; }
    int sms = 0;
    const int st = device_info(&sms);
    if (st != MLA_OK) return st;
    *ctas = (p->flags & MLA_FLAG_TCGEN05) ? sms : 2 * sms;
    return MLA_OK;
}

int check_header(const MlaDecodeParams* p) {
    if (!p || p->struct_size != sizeof(MlaDecodeParams) || p->abi_version != MLA_ABI_VERSION)
        return MLA_E_INVALID_ARG;
    if (p->heads != MLA_HEADS || p->qk_nope != MLA_QK_NOPE || p->qk_rope != MLA_QK_ROPE ||
        p->v_head != MLA_V_HEAD || p->kv_lora != MLA_KV_LORA || p->page_size != MLA_PAGE_SIZE)
        return MLA_E_UNSUPPORTED_DIMS;
    if (p->batch <= 0) return MLA_E_INVALID_ARG;
    if (p->batch > MLA_MAX_BATCH) return MLA_E_LIMIT;
    return MLA_OK;
}

// Full validation for the launch paths; fills `out` with num_ctas resolved.
int prepare(const MlaDecodeParams* p, MlaDecodeParams* out) {
    int st = check_header(p);
    if (st != MLA_OK) return st;
    const bool project = p->x_n != nullptr;
    if (project ? (p->q || p->kv_a || !p->w_qkv) : (!p->q || !p->kv_a)) return MLA_E_INVALID_ARG;
    if (!p->kv_a_norm_w || !p->kv_b || !p->rope_cos || !p->rope_sin || !p->block_table ||
        !p->seq_lens || !p->kv_cache || (!p->out && !p->shard_out) || !p->workspace)
        return MLA_E_INVALID_ARG;
    if (p->w_o) {  // K5 reads `out` back through a TMA map and writes h_out
        if (!p->out || p->shard_out || !p->residual || !p->h_out) return MLA_E_INVALID_ARG;
        if (p->residual_stride < MLA_HIDDEN || p->h_out_stride < MLA_HIDDEN) return MLA_E_INVALID_ARG;
        if (!aligned(p->out, 16) || (p->out_stride & 7) || !aligned(p->w_o, 16) || !aligned(p->residual, 8) ||
            (p->residual_stride & 3) || !aligned(p->h_out, 8) || (p->h_out_stride & 3))
            return MLA_E_MISALIGNED;
    }
    if (project) {
        if (p->x_stride < MLA_HIDDEN) return MLA_E_INVALID_ARG;
        if (!aligned(p->x_n, 16) || (p->x_stride & 7) || !aligned(p->w_qkv, 16)) return MLA_E_MISALIGNED;
    }
    if (p->flags & ~(MLA_FLAG_CHECK_KERNEL | MLA_FLAG_TCGEN05 | MLA_FLAG_NO_NEW_ROW | MLA_FLAG_EXCHANGE_SPLIT |
                     MLA_FLAG_QC_HILO | MLA_FLAG_P_HILO))
        return MLA_E_INVALID_ARG;
    if ((p->flags & (MLA_FLAG_QC_HILO | MLA_FLAG_P_HILO)) && (p->flags & (MLA_FLAG_CHECK_KERNEL | MLA_FLAG_TCGEN05)))
        return MLA_E_INVALID_ARG;  // the hi/lo forms exist in the default kernel only
    if (p->world < 0 || p->world > MLA_MAX_RANKS) return MLA_E_INVALID_ARG;
    if (p->world > 0) {  // peer exchange: K3 writes every rank's buffer, K4 combines into out
        if (p->rank < 0 || p->rank >= p->world || p->shard_out || !p->out || p->exchange_timeout_us < 0)
            return MLA_E_INVALID_ARG;
        if (p->exchange_batch < p->batch) return MLA_E_LIMIT;
        for (int r = 0; r < p->world; ++r) {
            if (!p->exchange[r]) return MLA_E_INVALID_ARG;
            if (!aligned(p->exchange[r], 256)) return MLA_E_MISALIGNED;
        }
    }
    if (p->max_blocks <= 0 || p->n_pages <= 0 || p->max_pos <= 0) return MLA_E_INVALID_ARG;
    if ((int64_t)p->n_pages * MLA_PAGE_SIZE > INT32_MAX || (int64_t)p->batch * p->max_blocks > INT32_MAX)
        return MLA_E_LIMIT;
    if ((!project && (p->q_stride < MLA_HEADS * (MLA_QK_NOPE + MLA_QK_ROPE) || p->kv_a_stride < MLA_ROW)) ||
        p->out_stride < MLA_HEADS * MLA_V_HEAD)
        return MLA_E_INVALID_ARG;
    if (!(p->softmax_scale > 0.f) || !(p->rms_eps >= 0.f)) return MLA_E_INVALID_ARG;
    if (!aligned(p->kv_cache, 16) || !aligned(p->kv_b, 16) || !aligned(p->workspace, 256) ||
        !aligned(p->q, 4) || (p->q_stride & 1) || (p->out_stride & 1) || !aligned(p->kv_a, 2) || !aligned(p->out, 4) || !aligned(p->kv_a_norm_w, 2) ||
        !aligned(p->rope_cos, 4) || !aligned(p->rope_sin, 4) || !aligned(p->rope_pos, 4) ||
        !aligned(p->shard_out, 16))
        return MLA_E_MISALIGNED;
    int sms = 0;
    st = device_info(&sms);
    if (st != MLA_OK) return st;
    *out = *p;
    if (p->error_host) {  // must be pinned host memory that the device can store into
        if (!aligned(p->error_host, 4)) return MLA_E_MISALIGNED;
        cudaPointerAttributes a;
        if (cudaPointerGetAttributes(&a, p->error_host) != cudaSuccess || a.type != cudaMemoryTypeHost ||
            !a.devicePointer) {
            cudaGetLastError();
            return MLA_E_INVALID_ARG;
        }
        out->error_host = static_cast<int32_t*>(a.devicePointer);
    }
    st = resolve_ctas(p, &out->num_ctas);
    if (st != MLA_OK) return st;
    const WsLayout ws = ws_layout(*out);
    if (p->workspace_bytes < ws.total) return MLA_E_WORKSPACE;
    if (project) {  // K1 onwards read the projection from the workspace
        const __nv_bfloat16* qkv =
            reinterpret_cast<const __nv_bfloat16*>(reinterpret_cast<const char*>(p->workspace) + ws.qkv);
        out->q = qkv;
        out->q_stride = kQkvRows;
        out->kv_a = qkv + kHeads * kQHead;
        out->kv_a_stride = kQkvRows;
    }
    return MLA_OK;
}

int run_exchange_combine(const MlaDecodeParams& q, cudaStream_t s) {
    return launch_exchange_combine(q, s) == cudaSuccess ? MLA_OK : MLA_E_LAUNCH;
}

int run_attention(const MlaDecodeParams& q, cudaStream_t s) {
    const float scale_log2 = (float)((double)q.softmax_scale * 1.4426950408889634);
    if (q.flags & MLA_FLAG_CHECK_KERNEL) {
        return launch_attention_check(q, scale_log2, s) == cudaSuccess ? MLA_OK : MLA_E_LAUNCH;
    }
    CUtensorMap tkv, tq;
    const bool tc = (q.flags & MLA_FLAG_TCGEN05) != 0;
    int st = make_tmap_blocks(&tkv, q.kv_cache, (uint64_t)q.n_pages, true, tc ? kPage : kPage / 2);
    if (st != MLA_OK) return st;
    if (!tc) {
        int sms = 0;
        st = device_info(&sms);
        if (st != MLA_OK) return st;
        return launch_attention_mma(q, tkv, scale_log2, sms, s) == cudaSuccess ? MLA_OK : MLA_E_LAUNCH;
    }
    const WsLayout ws = ws_layout(q);
    st = make_tmap_blocks(&tq, reinterpret_cast<const char*>(q.workspace) + ws.qa, (uint64_t)q.batch * kQRows, false,
                          kQRows);
    if (st != MLA_OK) return st;
    return launch_attention_tc(q, tkv, tq, scale_log2, s) == cudaSuccess ? MLA_OK : MLA_E_LAUNCH;
}

}  // namespace
}  // namespace mla

using namespace mla;

extern "C" {

int mla_abi_version(void) { return MLA_ABI_VERSION; }

const char* mla_status_string(int status) {
    switch (status) {
        case MLA_OK: return "MLA_OK";
        case MLA_E_INVALID_ARG: return "MLA_E_INVALID_ARG";
        case MLA_E_UNSUPPORTED_DIMS: return "MLA_E_UNSUPPORTED_DIMS";
        case MLA_E_MISALIGNED: return "MLA_E_MISALIGNED";
        case MLA_E_WORKSPACE: return "MLA_E_WORKSPACE";
        case MLA_E_ARCH: return "MLA_E_ARCH";
        case MLA_E_LAUNCH: return "MLA_E_LAUNCH";
        case MLA_E_DRIVER: return "MLA_E_DRIVER";
        case MLA_E_LIMIT: return "MLA_E_LIMIT";
        default: return "MLA_E_UNKNOWN";
    }
}

const char* mla_device_error_string(int code) {
    switch (code) {
        case MLA_DEV_OK: return "ok";
        case MLA_DEV_BAD_PAGE: return "block_table entry outside [0, n_pages)";
        case MLA_DEV_BAD_POSITION: return "seq_lens entry outside the rope table or block table";
        case MLA_DEV_TIMEOUT: return "on-chip pipeline wait timed out";
        case MLA_DEV_PEER_TIMEOUT: return "shard exchange: a peer's flag did not arrive in time";
        default: return "unknown device error";
    }
}

void mla_params_init(MlaDecodeParams* p) {
    if (!p) return;
    *p = MlaDecodeParams{};
    p->struct_size = sizeof(MlaDecodeParams);
    p->abi_version = MLA_ABI_VERSION;
    p->heads = MLA_HEADS;
    p->qk_nope = MLA_QK_NOPE;
    p->qk_rope = MLA_QK_ROPE;
    p->v_head = MLA_V_HEAD;
    p->kv_lora = MLA_KV_LORA;
    p->page_size = MLA_PAGE_SIZE;
    p->rms_eps = 1e-6f;
}

int mla_workspace_size(const MlaDecodeParams* p, uint64_t* bytes) {
    if (!bytes) return MLA_E_INVALID_ARG;
    int st = check_header(p);
    if (st != MLA_OK) return st;
    int ctas = 0;
    st = resolve_ctas(p, &ctas);
    if (st != MLA_OK) return st;
    *bytes = ws_layout(p->batch, ctas, p->x_n != nullptr, (p->flags & MLA_FLAG_QC_HILO) != 0).total;
    return MLA_OK;
}

int mla_plan_info(const MlaDecodeParams* p, int32_t* num_ctas, int32_t* num_slots) {
    int st = check_header(p);
    if (st != MLA_OK) return st;
    int ctas = 0;
    st = resolve_ctas(p, &ctas);
    if (st != MLA_OK) return st;
    if (num_ctas) *num_ctas = ctas;
    if (num_slots) *num_slots = ws_layout(p->batch, ctas, p->x_n != nullptr, (p->flags & MLA_FLAG_QC_HILO) != 0).slots;
    return MLA_OK;
}

int mla_launches_per_step(void) { return 3; }

int mla_combine_shards(const float* parts, int32_t n_shards, int32_t batch, void* out, int64_t out_stride,
                       void* stream) {
    if (!parts || !out || n_shards <= 0 || batch <= 0 || out_stride < MLA_HEADS * MLA_V_HEAD || (out_stride & 1))
        return MLA_E_INVALID_ARG;
    if (n_shards > 4096 || batch > MLA_MAX_BATCH) return MLA_E_LIMIT;
    if (!aligned(parts, 16) || !aligned(out, 4)) return MLA_E_MISALIGNED;
    const int st = device_info(nullptr);
    if (st != MLA_OK) return st;
    return launch_combine_shards(parts, n_shards, batch, out, out_stride, (cudaStream_t)stream) == cudaSuccess
               ? MLA_OK
               : MLA_E_LAUNCH;
}

void mla_rows_init(MlaRowsToPages* r) {
    if (!r) return;
    *r = MlaRowsToPages{};
    r->struct_size = sizeof(MlaRowsToPages);
    r->abi_version = MLA_ABI_VERSION;
    r->rms_eps = 1e-6f;
}

int mla_rows_to_pages(const MlaRowsToPages* r, void* stream) {
    if (!r || r->struct_size != sizeof(MlaRowsToPages) || r->abi_version != MLA_ABI_VERSION) return MLA_E_INVALID_ARG;
    if ((r->mode != MLA_ROWS_FINAL && r->mode != MLA_ROWS_RAW) || r->batch <= 0 || r->total_rows < 0 ||
        !r->row_start || !r->block_table || !r->kv_cache || r->max_blocks <= 0 || r->n_pages <= 0 ||
        r->rows_stride < MLA_ROW || (r->total_rows > 0 && !r->rows))
        return MLA_E_INVALID_ARG;
    if (r->batch > MLA_MAX_BATCH) return MLA_E_LIMIT;
    if (r->mode == MLA_ROWS_RAW && (!r->kv_a_norm_w || !r->rope_cos || !r->rope_sin || r->max_pos <= 0 ||
                                    !(r->rms_eps >= 0.f)))
        return MLA_E_INVALID_ARG;
    if (!aligned(r->rows, 16) || (r->rows_stride & 7) || !aligned(r->kv_cache, 16) || !aligned(r->row_start, 8) ||
        !aligned(r->kv_a_norm_w, 2) || !aligned(r->rope_cos, 4) || !aligned(r->rope_sin, 4))
        return MLA_E_MISALIGNED;
    int sms = 0;
    const int st = device_info(&sms);
    if (st != MLA_OK) return st;
    return launch_rows_to_pages(*r, sms, (cudaStream_t)stream) == cudaSuccess ? MLA_OK : MLA_E_LAUNCH;
}

int mla_project(const MlaDecodeParams* p, void* stream) {
    MlaDecodeParams q;
    int st = prepare(p, &q);
    if (st != MLA_OK) return st;
    if (!q.x_n) return MLA_E_INVALID_ARG;
    return run_project(q, (cudaStream_t)stream);
}

int mla_o_proj(const MlaDecodeParams* p, void* stream) {
    MlaDecodeParams q;
    int st = prepare(p, &q);
    if (st != MLA_OK) return st;
    if (!q.w_o) return MLA_E_INVALID_ARG;
    return run_o_proj(q, (cudaStream_t)stream);
}

int mla_prologue(const MlaDecodeParams* p, void* stream) {
    MlaDecodeParams q;
    int st = prepare(p, &q);
    if (st != MLA_OK) return st;
    return run_prologue(q, (cudaStream_t)stream);
}

int mla_attention(const MlaDecodeParams* p, void* stream) {
    MlaDecodeParams q;
    int st = prepare(p, &q);
    if (st != MLA_OK) return st;
    return run_attention(q, (cudaStream_t)stream);
}

int mla_merge_uv(const MlaDecodeParams* p, void* stream) {
    MlaDecodeParams q;
    int st = prepare(p, &q);
    if (st != MLA_OK) return st;
    return run_merge(q, (cudaStream_t)stream);
}

int mla_exchange_combine(const MlaDecodeParams* p, void* stream) {
    MlaDecodeParams q;
    int st = prepare(p, &q);
    if (st != MLA_OK) return st;
    if (q.world <= 0) return MLA_E_INVALID_ARG;
    return run_exchange_combine(q, (cudaStream_t)stream);
}

int mla_decode_step(const MlaDecodeParams* p, void* stream) {
    MlaDecodeParams q;
    int st = prepare(p, &q);
    if (st != MLA_OK) return st;
    cudaStream_t s = (cudaStream_t)stream;
    if (q.x_n) {
        st = run_project(q, s);
        if (st != MLA_OK) return st;
    }
    st = run_prologue(q, s);
    if (st != MLA_OK) return st;
    st = run_attention(q, s);
    if (st != MLA_OK) return st;
    const bool fused = exchange_fused(q);
    st = run_merge(q, s, fused);
    if (st != MLA_OK) return st;
    if (q.world > 0 && !fused) {
        st = run_exchange_combine(q, s);
        if (st != MLA_OK) return st;
    }
    return q.w_o ? run_o_proj(q, s) : MLA_OK;
}

int mla_exchange_bytes(int32_t world, int32_t max_batch, uint64_t* bytes) {
    if (!bytes || world <= 0 || max_batch <= 0) return MLA_E_INVALID_ARG;
    if (world > MLA_MAX_RANKS || max_batch > MLA_MAX_BATCH) return MLA_E_LIMIT;
    *bytes = ex_layout(world, max_batch).total;
    return MLA_OK;
}

int mla_exchange_alloc(uint64_t bytes, void** buf, void* ipc_handle) {
    if (!buf || bytes == 0) return MLA_E_INVALID_ARG;
    *buf = nullptr;
    const int st = device_info(nullptr);
    if (st != MLA_OK) return st;
    void* ptr = nullptr;
    if (cudaMalloc(&ptr, bytes) != cudaSuccess) return MLA_E_LAUNCH;
    if (cudaMemset(ptr, 0, bytes) != cudaSuccess || cudaDeviceSynchronize() != cudaSuccess) {
        cudaFree(ptr);
        return MLA_E_LAUNCH;
    }
    if (ipc_handle) {
        cudaIpcMemHandle_t h;
        static_assert(sizeof(h) == MLA_IPC_HANDLE_BYTES, "IPC handle size");
        if (cudaIpcGetMemHandle(&h, ptr) != cudaSuccess) {
            cudaFree(ptr);
            return MLA_E_LAUNCH;
        }
        memcpy(ipc_handle, &h, sizeof(h));
    }
    *buf = ptr;
    return MLA_OK;
}

int mla_exchange_free(void* buf) {
    if (!buf) return MLA_E_INVALID_ARG;
    return cudaFree(buf) == cudaSuccess ? MLA_OK : MLA_E_LAUNCH;
}

int mla_exchange_open(const void* ipc_handle, void** buf) {
    if (!ipc_handle || !buf) return MLA_E_INVALID_ARG;
    *buf = nullptr;
    const int st = device_info(nullptr);
    if (st != MLA_OK) return st;
    cudaIpcMemHandle_t h;
    memcpy(&h, ipc_handle, sizeof(h));
    void* ptr = nullptr;
    if (cudaIpcOpenMemHandle(&ptr, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) return MLA_E_LAUNCH;
    *buf = ptr;
    return MLA_OK;
}

int mla_exchange_close(void* buf) {
    if (!buf) return MLA_E_INVALID_ARG;
    return cudaIpcCloseMemHandle(buf) == cudaSuccess ? MLA_OK : MLA_E_LAUNCH;
}

}  // extern "C"

