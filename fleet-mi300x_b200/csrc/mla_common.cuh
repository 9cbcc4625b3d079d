// Shared device helpers for the MLA decode kernels (sm_100a only).
//
// PTX wrappers for mbarriers, TMA (cp.async.bulk.tensor, no multicast),
// tcgen05 (MMA, TMEM alloc/ld/st, commit, fences), bounded waits and the
// workspace layout shared by the host glue and the three kernels.
#pragma once

#include <cuda_runtime.h>
#include <utility>
#include <cuda_bf16.h>
#include <stdint.h>

#include "mla_decode.h"

namespace mla {

constexpr int kHeads = MLA_HEADS;          // 16
constexpr int kNope = MLA_QK_NOPE;         // 128
constexpr int kRope = MLA_QK_ROPE;         // 64
constexpr int kV = MLA_V_HEAD;             // 128
constexpr int kLora = MLA_KV_LORA;         // 512
constexpr int kRow = MLA_ROW;              // 576
constexpr int kPage = MLA_PAGE_SIZE;       // 64
constexpr int kQHead = kNope + kRope;      // 192: q row per head
constexpr int kKvbHead = kNope + kV;       // 256: kv_b rows per head
constexpr int kQRows = kHeads;             // rows of the absorbed query per request in the workspace
constexpr int kHidden = MLA_HIDDEN;        // 2048: model width (x_n)
constexpr int kQkvRows = kHeads * kQHead + kRow;  // 3648: rows of the stacked [W_q; W_kv_a]
constexpr int kK1LatQ = 128;               // latent columns of W_UK per prologue CTA (a quarter)
constexpr int kK1WukBlocks = kK1LatQ / 64; // 64-column blocks of that slice (its TMA box)
constexpr float kLog2e = 1.4426950408889634f;

// ---------------------------------------------------------------------------
// Workspace layout (bytes, each region 256-byte aligned).
//   tiles_cum  int32 [batch + 1]          prefix sum of plan tiles per request (plan_unit_rows)
//   plan       PlanHeader, PlanEntry [num_ctas]   the split plan per CTA, ready to use (K1 writes it)
//   qa         bf16  [batch][16][576]     absorbed query q_c (512) | roped q_pe (64), per head
//   part_ml    f32   [slots][16][2]       split partial: running max (log2 domain), sum of exps
//   part_acc   f32   [slots][16][512]     split partial: unnormalised sum_t p_t * c_t
//   qkv        bf16  [batch][3648]        q | kv_a, when the step projects x_n itself (K0)
//   qa_lo      bf16  [batch][16][512]     q_c - bf16(q_c), with MLA_FLAG_QC_HILO
// slots = num_ctas + batch: CTA c writes the partial of request b at slot c + b.
// ---------------------------------------------------------------------------
struct WsLayout {
    uint64_t tiles_cum, plan, qa, part_ml, part_acc, qkv, qa_lo, total;
    int32_t slots;
};

// The split plan as K1's planner leaves it for the split-KV kernel: the total tile
// count U, the number of CTAs with work G = min(U, num_ctas), and per plan CTA its
// tile range, its first request b (the largest b with cum[b] <= u_begin) and that
// request's cum[b], cum[b + 1], so that the kernel starts without a search.
struct PlanHeader {
    int64_t U;
    int32_t G, pad;
};
struct PlanEntry {
    int64_t u_begin, u_end;
    int32_t b, cb0, cb1, pad;
};

__host__ __device__ inline uint64_t align256(uint64_t x) { return (x + 255) & ~uint64_t(255); }

// with_qkv: the step projects x_n itself (MlaDecodeParams.x_n set), and q | kv_a
// of every request live in the workspace as [batch][3648] bf16.
// with_qlo: MLA_FLAG_QC_HILO, the low half of q_c lives in qa_lo.
__host__ __device__ inline WsLayout ws_layout(int batch, int num_ctas, bool with_qkv = false, bool with_qlo = false) {
    WsLayout w;
    w.slots = num_ctas + batch;
    uint64_t off = 0;
    w.tiles_cum = off; off = align256(off + uint64_t(batch + 1) * 4);
    w.plan = off;      off = align256(off + sizeof(PlanHeader) + uint64_t(num_ctas) * sizeof(PlanEntry));
    w.qa = off;        off = align256(off + uint64_t(batch) * kQRows * kRow * 2);
    w.part_ml = off;   off = align256(off + uint64_t(w.slots) * kHeads * 2 * 4);
    w.part_acc = off;  off = align256(off + uint64_t(w.slots) * kHeads * kLora * 4);
    w.qkv = off;       off = align256(off + (with_qkv ? uint64_t(batch) * kQkvRows * 2 : 0));
    w.qa_lo = off;     off = align256(off + (with_qlo ? uint64_t(batch) * kQRows * kLora * 2 : 0));
    w.total = off;
    return w;
}

__host__ __device__ inline WsLayout ws_layout(const MlaDecodeParams& p) {
    return ws_layout(p.batch, p.num_ctas, p.x_n != nullptr, (p.flags & MLA_FLAG_QC_HILO) != 0);
}


// The split-KV kernel's grid for num_ctas plan CTAs (two warp groups per CTA, each
// one plan CTA): up to one CTA per SM with one group each, then a second group in
// the same CTAs; beyond two per SM, CTAs of two groups each.
inline int k2_grid(int num_ctas, int sm_count) {
    const int two = (num_ctas + 1) / 2;
    return num_ctas <= sm_count ? num_ctas : (two > sm_count ? two : sm_count);
}

// Pair merge. When every CTA of the split-KV kernel runs two plan CTAs and the plan
// has num_ctas CTAs (G = num_ctas: at least num_ctas tiles), the two are made
// adjacent (2k, 2k + 1). Where their boundary falls inside a request, group 1's
// first partial (that request's) is merged in shared memory into group 0's last one
// (slot 2k + b), so that K3 folds fewer partials: a request's partials then sit at
// its first plan CTA and at every even plan CTA after it. Both kernels take this
// flag from the host and test G themselves. Only the default (mma) split-KV kernel
// pairs.
inline bool k2_pairs(const MlaDecodeParams& p, int sm_count) {
    return (p.flags & (MLA_FLAG_CHECK_KERNEL | MLA_FLAG_TCGEN05)) == 0 && p.num_ctas % 2 == 0 &&
           2 * k2_grid(p.num_ctas, sm_count) == p.num_ctas;
}

// Programmatic dependent launch. A kernel launched with launch_pdl may start
// while the kernel before it on the stream is still running; pdl_wait() returns
// once that kernel has completed and its writes are visible, so it must come
// before any read of data an earlier kernel writes and before any write an
// earlier kernel may still read. pdl_trigger() lets the next PDL kernel launch
// as soon as every CTA of this one has issued it. Both are no-ops for a kernel
// launched without the attribute.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                              Args&&... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// Split plan: the CTA grid shares the flattened list of tiles of all requests
// evenly. CTA c owns tiles [c*U/G, (c+1)*U/G).
__host__ __device__ inline int64_t plan_begin(int c, int64_t U, int G) {
    return (int64_t)c * U / G;
}
// The CTA whose range holds tile u.
__host__ __device__ inline int plan_cta_of(int64_t u, int64_t U, int G) {
    return (int)(((u + 1) * (int64_t)G - 1) / U);
}

// ---------------------------------------------------------------------------
// Per-request positions. The new token's row is stored at local row seq_lens[b]
// and attended unless MLA_FLAG_NO_NEW_ROW (a sequence shard that does not own
// it); its RoPE position is rope_pos[b] when given (the global position of a
// sequence-sharded step), else seq_lens[b].
// ---------------------------------------------------------------------------
__host__ __device__ inline int new_row_count(const MlaDecodeParams& p) {
    return (p.flags & MLA_FLAG_NO_NEW_ROW) ? 0 : 1;
}
__device__ __forceinline__ int rope_position(const MlaDecodeParams& p, int b) {
    return p.rope_pos ? p.rope_pos[b] : p.seq_lens[b];
}

// Request b is valid if its RoPE position lies in the tables and its rows
// (cached + the new one, if this call stores it) fit its block-table row.
__device__ __forceinline__ bool request_ok(const MlaDecodeParams& p, int b) {
    const int rows = p.seq_lens[b], rp = rope_position(p, b);
    return rows >= 0 && rp >= 0 && rp < p.max_pos && rows + new_row_count(p) <= p.max_blocks * kPage;
}

// Rows per tile of the split plan: the default split-KV kernel walks 32-row half
// pages (its TMA box), the CUDA-core and tensor-memory kernels whole 64-row pages.
__host__ __device__ inline int plan_unit_rows(const MlaDecodeParams& p) {
    return (p.flags & (MLA_FLAG_CHECK_KERNEL | MLA_FLAG_TCGEN05)) ? kPage : kPage / 2;
}

// Tiles request b attends in the split plan: 0 for an invalid request (K1's
// planner records it), so that no kernel reads outside the block table.
__device__ __forceinline__ int plan_tiles(const MlaDecodeParams& p, int b) {
    const int unit = plan_unit_rows(p);
    return request_ok(p, b) ? (p.seq_lens[b] + new_row_count(p) + unit - 1) / unit : 0;
}

// ---------------------------------------------------------------------------
// Device errors. A kernel reports into the caller's device word (first error
// wins, by atomicCAS) and, if the caller gave one, into a pinned host word
// (MlaDecodeParams.error_host), which receives the winning code by a plain
// store over the system bus, so that the host sees the error without
// synchronising with the stream. Only error paths touch either word.
// ---------------------------------------------------------------------------
struct ErrSink {
    int32_t* dev;
    int32_t* host;
};

__host__ __device__ inline ErrSink err_sink(const MlaDecodeParams& p) { return ErrSink{p.error_word, p.error_host}; }

// Arguments of the tensor-core projection (mla_project_tc.cu): y[b][n] = epi(sum_k
// x[b][k] W[n][k]) for n < n_rows, b < batch; epi adds the residual for o_proj.
struct GemmArgs {
    __nv_bfloat16* y;
    int64_t y_stride;
    const __nv_bfloat16* residual;  // o_proj + residual only
    int64_t res_stride;
    int batch, n_rows;
    ErrSink err;
};

__device__ __forceinline__ void record_error(const ErrSink& e, int code) {
    int won = code;
    if (e.dev) {
        const int old = atomicCAS(e.dev, 0, code);
        if (old) won = old;
    }
    if (e.host) {
        *reinterpret_cast<volatile int32_t*>(e.host) = won;
        __threadfence_system();
    }
}

// ---------------------------------------------------------------------------
// Shared-memory addresses, mbarriers.
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}\n"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Non-blocking probe of one phase (never suspends the thread).
__device__ __forceinline__ bool mbar_test_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}\n"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// ---------------------------------------------------------------------------
// Exchange buffer of the peer-memory shard exchange (MlaDecodeParams.world > 0),
// one per rank, written by every rank's K3 and read by this rank's K4:
//   ctl    u32   [2]        steps completed by this rank's K4, K4 blocks done
//   lines  u64x2 [2][world][max_batch][16][kExLines]
//          the shard partial of (source rank, request, head) at parity = step & 1:
//          line j < 64 holds y[2j], y[2j+1]; line 64 holds m, L. Each 8-byte half of
//          a line is (step << 32) | f32 bits, stored and loaded as one 64-bit access,
//          so a reader that sees this step's number in a half also sees its value;
//          no flag or fence orders the data (the low-latency line format NCCL uses).
// ---------------------------------------------------------------------------
constexpr int kMaxRanks = MLA_MAX_RANKS;
constexpr int kK3ClusterCtas = 4;   // K3 cluster form: CTAs per (head, block of 16 requests)
constexpr int kExLines = kV / 2 + 1;  // 65 lines of 16 bytes per (source, request, head)

struct ExLayout {
    uint64_t ctl, lines, total;
};

__host__ __device__ inline ExLayout ex_layout(int world, int max_batch) {
    ExLayout e;
    uint64_t off = 0;
    e.ctl = off;   off = align256(off + 8);
    e.lines = off; off = align256(off + 2ull * world * max_batch * kHeads * kExLines * 16);
    e.total = off;
    return e;
}

// p.exchange[r] without a dynamically indexed parameter array (which would copy
// the whole parameter block to local memory).
__device__ __forceinline__ char* ex_buf(const MlaDecodeParams& p, int r) {
    char* b = nullptr;
#pragma unroll
    for (int d = 0; d < kMaxRanks; ++d)
        if (d == r) b = reinterpret_cast<char*>(p.exchange[d]);
    return b;
}

// First line of (source src, request b, head h) at parity par in an exchange buffer.
__device__ __forceinline__ ulonglong2* ex_lines(char* buf, const ExLayout& ex, int world, int max_batch,
                                                uint32_t par, int src, int b, int h) {
    return reinterpret_cast<ulonglong2*>(buf + ex.lines) +
           ((((int64_t)par * world + src) * max_batch + b) * kHeads + h) * kExLines;
}

// One line: two f32 values, each tagged with the step number in its 64-bit half.
__device__ __forceinline__ void st_line(ulonglong2* line, float a, float b, uint32_t step) {
    const unsigned long long x = ((unsigned long long)step << 32) | __float_as_uint(a);
    const unsigned long long y = ((unsigned long long)step << 32) | __float_as_uint(b);
    asm volatile("st.relaxed.sys.global.v2.b64 [%0], {%1, %2};" ::"l"(line), "l"(x), "l"(y) : "memory");
}

// One load of a line (both halves in one 128-bit access of two 64-bit elements).
__device__ __forceinline__ ulonglong2 ld_line(const ulonglong2* line) {
    ulonglong2 v;
    asm volatile("ld.relaxed.sys.global.v2.b64 {%0, %1}, [%2];" : "=l"(v.x), "=l"(v.y) : "l"(line) : "memory");
    return v;
}
__device__ __forceinline__ bool line_ready(const ulonglong2& v, uint32_t step) {
    return (uint32_t)(v.x >> 32) == step && (uint32_t)(v.y >> 32) == step;
}

// Wait until a line carries `step`, starting from an already loaded value v
// (true; v then holds the line) or until limit_ns have passed since t0 (false).
// Callers load all the lines they need first, so that one round trip serves them
// all when the data is already there.
__device__ __forceinline__ bool wait_line(const ulonglong2* line, uint32_t step, ulonglong2& v, uint64_t t0,
                                          uint64_t limit_ns) {
    for (uint32_t k = 1; !line_ready(v, step); ++k) {
        if ((k & 31) == 0 && globaltimer_ns() - t0 > limit_ns) return false;
        __nanosleep(32);
        v = ld_line(line);
    }
    return true;
}
__device__ __forceinline__ float line_lo(const ulonglong2& v) { return __uint_as_float((uint32_t)v.x); }
__device__ __forceinline__ float line_hi(const ulonglong2& v) { return __uint_as_float((uint32_t)v.y); }

// A wait on one phase of an mbarrier that gives up after `kWaitLimitNs` or
// when another role raised `*abort`. On giving up it records
// MLA_DEV_TIMEOUT, raises *abort and returns false. The limit is per wait: a
// healthy pipeline completes each phase in microseconds.
constexpr uint64_t kWaitLimitNs = 1500ull * 1000ull * 1000ull;  // 1.5 s

__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, volatile int* abort,
                                          const ErrSink& err) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = globaltimer_ns();
    for (uint32_t i = 1;; ++i) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((i & 63) == 0) {
            if (*abort) return false;
            if (globaltimer_ns() - t0 > kWaitLimitNs) {
                record_error(err, MLA_DEV_TIMEOUT);
                *abort = 1;
                return false;
            }
        }
    }
}

__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void named_bar_sync(int id, int nthreads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// Named barrier that also ORs a predicate over the participating threads.
__device__ __forceinline__ bool bar_red_or(int id, int nthreads, bool pred) {
    uint32_t r;
    asm volatile(
        "{\n\t.reg .pred p, q;\n\t"
        "setp.ne.u32 p, %1, 0;\n\t"
        "bar.red.or.pred q, %2, %3, p;\n\t"
        "selp.u32 %0, 1, 0, q;\n\t}\n"
        : "=r"(r)
        : "r"((uint32_t)pred), "r"(id), "r"(nthreads)
        : "memory");
    return r != 0;
}

// ---------------------------------------------------------------------------
// Thread-block cluster primitives (sm_90+): this CTA's rank, a cluster-wide
// barrier with release/acquire ordering of shared memory, the cluster address of
// a shared-memory location in a peer CTA, and stores into it that complete their
// bytes on an mbarrier there (distributed shared memory; no global memory).
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t cluster_rank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
__device__ __forceinline__ void cluster_sync_all() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ uint32_t dsmem_addr(uint32_t smem_addr, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_addr), "r"(rank));
    return r;
}
__device__ __forceinline__ void dsmem_push4(uint32_t addr, float4 v, uint32_t remote_bar) {
    asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.v4.f32 [%0], {%1, %2, %3, %4}, [%5];"
                 ::"r"(addr), "f"(v.x), "f"(v.y), "f"(v.z), "f"(v.w), "r"(remote_bar) : "memory");
}
__device__ __forceinline__ void dsmem_push2(uint32_t addr, float2 v, uint32_t remote_bar) {
    asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.v2.f32 [%0], {%1, %2}, [%3];"
                 ::"r"(addr), "f"(v.x), "f"(v.y), "r"(remote_bar) : "memory");
}

// ---------------------------------------------------------------------------
// TMA: tiled loads global -> shared, completion on an mbarrier. Never with
// cluster multicast.
// ---------------------------------------------------------------------------
constexpr uint64_t kCacheEvictFirst = 0x12F0000000000000ull;
constexpr uint64_t kCacheEvictLast = 0x14F0000000000000ull;

__device__ __forceinline__ void tma_load_3d(void* smem_dst, const void* tmap, uint64_t* bar, int x, int y, int z,
                                            uint64_t cache_hint) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
        " [%0], [%1, {%3, %4, %5}], [%2], %6;" ::"r"(smem_u32(smem_dst)),
        "l"(reinterpret_cast<uint64_t>(tmap)), "r"(smem_u32(bar)), "r"(x), "r"(y), "r"(z), "l"(cache_hint)
        : "memory");
}

__device__ __forceinline__ void tma_load_4d(void* smem_dst, const void* tmap, uint64_t* bar, int x, int y, int z,
                                            int w, uint64_t cache_hint) {
    asm volatile(
        "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
        " [%0], [%1, {%3, %4, %5, %6}], [%2], %7;" ::"r"(smem_u32(smem_dst)),
        "l"(reinterpret_cast<uint64_t>(tmap)), "r"(smem_u32(bar)), "r"(x), "r"(y), "r"(z), "r"(w), "l"(cache_hint)
        : "memory");
}

__device__ __forceinline__ void prefetch_tmap(const void* tmap) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(tmap)) : "memory");
}

// ---------------------------------------------------------------------------
// tcgen05: tensor memory and the 5th-generation MMA.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void tmem_alloc(uint32_t* smem_result, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(smem_result)),
                 "r"(ncols)
                 : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// D(tmem) (+)= A(smem desc) * B(smem desc), kind::f16 (bf16 in, fp32 accumulate).
__device__ __forceinline__ void tc_mma_f16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                           uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// Make the mbarrier track completion of every tcgen05 op this thread issued so far.
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                     smem_u32(bar))
                 : "memory");
}

// 32 lanes x 32 bits, 16 consecutive columns: thread i of the warp gets lane
// (warp's subpartition base + i), columns [col, col+16).
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
    uint32_t r[16];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
        "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ void tmem_st16(uint32_t taddr, const float (&v)[16]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
        "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16};" ::"r"(taddr),
        "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])),
        "r"(__float_as_uint(v[3])), "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])),
        "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])), "r"(__float_as_uint(v[8])),
        "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])), "r"(__float_as_uint(v[11])),
        "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])), "r"(__float_as_uint(v[14])),
        "r"(__float_as_uint(v[15]))
        : "memory");
}

__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// Shared-memory matrix descriptor (tcgen05 "version 1" layout):
//   [0,14) start >> 4, [16,30) leading byte offset >> 4, [32,46) stride byte
//   offset >> 4, [46,48) version = 1, [49,52) base offset = 0, [61,64) layout
//   (2 = 128-byte swizzle). Every swizzle atom used here is 1024-byte aligned.
__device__ __forceinline__ uint64_t smem_desc_sw128(uint32_t saddr, uint32_t lbo_bytes, uint32_t sbo_bytes) {
    uint64_t d = 0;
    d |= uint64_t((saddr >> 4) & 0x3FFF);
    d |= uint64_t((lbo_bytes >> 4) & 0x3FFF) << 16;
    d |= uint64_t((sbo_bytes >> 4) & 0x3FFF) << 32;
    d |= uint64_t(1) << 46;
    d |= uint64_t(2) << 61;
    return d;
}

// Instruction descriptor of kind::f16 with bf16 A/B and fp32 D.
//   [4,6) D format (1 = f32), [7,10) A format (1 = bf16), [10,13) B format,
//   [15] A major (0 = K, 1 = MN), [16] B major, [17,23) N >> 3, [24,29) M >> 4.
__host__ __device__ constexpr uint32_t idesc_bf16_f32(int M, int N, int a_mn_major, int b_mn_major) {
    return (1u << 4) | (1u << 7) | (1u << 10) | (uint32_t(a_mn_major) << 15) | (uint32_t(b_mn_major) << 16) |
           (uint32_t(N >> 3) << 17) | (uint32_t(M >> 4) << 24);
}

// ---------------------------------------------------------------------------
// Small math helpers.
// ---------------------------------------------------------------------------
__device__ __forceinline__ float bf16_round(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

__device__ __forceinline__ float fast_exp2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// ---------------------------------------------------------------------------
// Optional per-tile trace stamps (SM clock), compiled in only with -DMLA_TRACE:
// the role timeline of the attention kernel, read back by mla_trace_read().
// ---------------------------------------------------------------------------
#ifdef MLA_TRACE
constexpr int kTraceCtas = 160, kTraceTiles = 96, kTraceEvents = 8;
// g_mla_trace is defined in mla_attention.cu, the only translation unit that stamps.
#define MLA_STAMP(tile, ev)                                                                          \
    do {                                                                                             \
        if (blockIdx.x < ::mla::kTraceCtas && (tile) < ::mla::kTraceTiles)                           \
            ::mla::g_mla_trace[((int)blockIdx.x * ::mla::kTraceTiles + (tile)) * ::mla::kTraceEvents + \
                               (ev)] = clock64();                                                    \
    } while (0)
#else
#define MLA_STAMP(tile, ev) \
    do {                    \
    } while (0)
#endif

// Optional kernel timeline (trace build only): per kernel and CTA, %globaltimer at
// entry (thread 0), after pdl_wait (thread 0) and at exit (the last warp of the CTA
// to return), the SM id, and two kernel-specific marks (latest writer wins); read
// back by mla_timeline_read(). Kernels: 0 = K1, 1 = K2, 2 = K3, 3 = K4, 4 = K0 / K5.
#ifdef MLA_TRACE
constexpr int kTlKernels = 5, kTlCtas = 512, kTlEvents = 6;
extern __device__ unsigned long long g_mla_timeline[kTlKernels * kTlCtas * kTlEvents];
__device__ __forceinline__ void tl_stamp(int k, int ev) {
    const int cta = (int)(blockIdx.y * gridDim.x + blockIdx.x);
    if (cta >= kTlCtas) return;
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    unsigned long long* slot = &g_mla_timeline[(k * kTlCtas + cta) * kTlEvents];
    if (ev == 2) {
        if ((threadIdx.x & 31) == 0) atomicMax(slot + 2, t);
    } else if (threadIdx.x == 0) {
        slot[ev] = t;
        if (ev == 0) {
            unsigned sm;
            asm volatile("mov.u32 %0, %%smid;" : "=r"(sm));
            slot[3] = sm + 1;
        }
    }
}
struct TlScope {  // entry stamp now, exit stamp on every return path
    int k;
    __device__ explicit TlScope(int kernel) : k(kernel) { tl_stamp(k, 0); }
    __device__ ~TlScope() { tl_stamp(k, 2); }
};
__device__ __forceinline__ void tl_mark(int k, int slot) {  // slot 4 or 5; lane 0 of the calling warp
    const int cta = (int)(blockIdx.y * gridDim.x + blockIdx.x);
    if (cta >= kTlCtas || (threadIdx.x & 31) != 0) return;
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    atomicMax(&g_mla_timeline[(k * kTlCtas + cta) * kTlEvents + slot], t);
}
#define MLA_TL_SCOPE(k) ::mla::TlScope mla_tl_scope_(k)
#define MLA_TL_WAITED(k) ::mla::tl_stamp(k, 1)
#define MLA_TL_MARK(k, slot) ::mla::tl_mark(k, slot)
#else
#define MLA_TL_MARK(k, slot) \
    do {                     \
    } while (0)
#define MLA_TL_SCOPE(k) \
    do {                \
    } while (0)
#define MLA_TL_WAITED(k) \
    do {                 \
    } while (0)
#endif

}  // namespace mla
