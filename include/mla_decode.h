/*
 * mla_decode.h — C ABI of the B200 (sm_100a) absorbed-MLA decode-attention path.
 *
 * This library is a drop-in for the attention task of the reference's
 * task-by-task decode: reference_decode.py:attention_absorbed
 * (src/host/reference_decode.py:210-256), restricted to the slice between the
 * input RMSNorm (:222) and o_proj (:256). Inputs are either the post-RMSNorm
 * hidden state x_n with the stacked [W_q; W_kv_a] weight (the library then
 * projects q and kv_a itself, :225-231), or the q / kv_a projections; the
 * output is the head-concatenated, bf16-rounded attention result R(out)
 * before o_proj (:256).
 *
 * On the device the reference runs this slice as three task kinds inside its
 * persistent kernel (src/kernels/fleet_kernel.hip:647-654 TASK_Q_ABSORB,
 * :745-798 TASK_ATTENTION, :694-701 TASK_MERGE_UV), launched through
 * `extern "C" hipError_t fleet_launch_step(...)` (fleet_kernel.hip:1068-1078).
 * Here the same work is three stream-ordered kernels (up to five, with the
 * q | kv_a projection before and o_proj + residual after) behind plain C entry
 * points: pointers, sizes and a caller-provided workspace; no allocation, no
 * torch types, no global mutable state except a per-device attribute cache.
 *
 * Layouts (all device memory, row-major):
 *   q            bf16 [batch][q_stride]      head h: [192h, 192h+128) q_nope, [192h+128, 192h+192) q_pe
 *   kv_a         bf16 [batch][kv_a_stride]   [0,512) c_new (raw), [512,576) k_pe_new (raw)
 *   kv_a_norm_w  bf16 [512]                  kv_a_layernorm.weight
 *   kv_b         bf16 [16*256][512]          kv_b_proj.weight: head h rows [256h,256h+128) = W_UK,
 *                                            [256h+128, 256h+256) = W_UV (reference_decode.py:242-248)
 *   rope_cos/sin f32  [max_pos][64]          YaRN tables (reference_decode.py:102-117)
 *   kv_cache     bf16 [n_pages][64][576]     paged latent cache: row = c_kv(512) | k_pe(64)
 *   block_table  i32  [batch][max_blocks]    page ids of each request's logical pages
 *   seq_lens     i32  [batch]                rows cached before this step = position of the new token
 *   out          bf16 [batch][out_stride]    R(out): head h at [128h, 128h+128)
 *
 * One call appends each request's new row at position seq_lens[b] (the
 * reference's in-place `cache[pos] = ...`, reference_decode.py:236-237) and
 * attends over rows 0..seq_lens[b] inclusive. It does not advance seq_lens;
 * the caller does, exactly as the reference's caller advances `pos`.
 */
#ifndef MLA_DECODE_H_
#define MLA_DECODE_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define MLA_ABI_VERSION 6

/* Fixed model dimensions. The reference's launcher refuses any other shape
 * (src/host/fleet_launch.hip:573-577: kv_lora != 512 or qk_rope != 64);
 * these kernels refuse the same way, with MLA_E_UNSUPPORTED_DIMS. */
#define MLA_HEADS 16
#define MLA_QK_NOPE 128
#define MLA_QK_ROPE 64
#define MLA_V_HEAD 128
#define MLA_KV_LORA 512
#define MLA_PAGE_SIZE 64
#define MLA_ROW (MLA_KV_LORA + MLA_QK_ROPE)
#define MLA_HIDDEN 2048                                     /* model width: x_n rows */
#define MLA_QKV_ROWS (MLA_HEADS * (MLA_QK_NOPE + MLA_QK_ROPE) + MLA_ROW)  /* 3648: [W_q; W_kv_a] */
#define MLA_MAX_PROJECT_BATCH 64                            /* the projections of batches up to this stream their
                                                               weight (m16n8k16); larger batches run a tcgen05 GEMM */
#define MLA_MAX_RANKS 8                                     /* shards of a step with the peer exchange */
#define MLA_IPC_HANDLE_BYTES 64                             /* size of an exchange buffer's IPC handle */

/* Host-side status codes (return values). The reference's launcher dies with
 * a message on bad shapes (fleet_launch.hip:573-577) and returns hipError_t
 * from the launch (fleet_kernel.hip:1068-1078); here every entry point
 * returns one of these instead of exiting. */
typedef enum {
    MLA_OK = 0,
    MLA_E_INVALID_ARG = -1,      /* null pointer, bad struct size/version, batch <= 0 */
    MLA_E_UNSUPPORTED_DIMS = -2, /* dims other than 16/128/64/128/512, page size != 64 */
    MLA_E_MISALIGNED = -3,       /* a pointer or stride breaks the 16-byte rule of TMA/vector loads */
    MLA_E_WORKSPACE = -4,        /* workspace missing or smaller than mla_workspace_size() */
    MLA_E_ARCH = -5,             /* current device is not sm_100 */
    MLA_E_LAUNCH = -6,           /* a CUDA launch/attribute call failed */
    MLA_E_DRIVER = -7,           /* cuTensorMapEncodeTiled unavailable or failed */
    MLA_E_LIMIT = -8             /* a size exceeds a documented limit (batch, pages, positions) */
} mla_status;

/* Device-side error codes, written to *error_word (first error wins, by
 * atomicCAS). The reference decodes its abort word the same way
 * (fleet_runtime.h:194-198, describe_abort in fleet_launch.hip:284-311). */
#define MLA_DEV_OK 0
#define MLA_DEV_BAD_PAGE 1      /* block_table entry outside [0, n_pages) */
#define MLA_DEV_BAD_POSITION 2  /* seq_lens[b] >= max_pos or >= max_blocks * 64, or < 0 */
#define MLA_DEV_TIMEOUT 3       /* a bounded on-chip wait gave up (pipeline stall) */
#define MLA_DEV_PEER_TIMEOUT 4  /* the exchange combine gave up waiting for a shard's flag
                                   (a peer that did not run its step within exchange_timeout_us) */

/* Flags. */
#define MLA_FLAG_CHECK_KERNEL 0x2 /* run the CUDA-core split-KV kernel instead of the tensor-core one
                                     (same plan and partial layout, fp32 probabilities; it exists to
                                     cross-check the tensor-core kernels, not as a fallback) */
#define MLA_FLAG_TCGEN05 0x4      /* run the split-KV kernel that keeps scores and the output in tensor
                                     memory (tcgen05.mma, tokens on M, heads on N) instead of the default
                                     m16n8k16 kernel (heads on M); same plan and partial layout */
#define MLA_FLAG_NO_NEW_ROW 0x8   /* sequence-sharded decode, a shard that does not own the new token:
                                     store no row and attend over cache rows 0..seq_lens[b]-1 only */
#define MLA_FLAG_EXCHANGE_SPLIT 0x10 /* peer exchange (world > 0): run it as K3 + K4 even where the fused
                                        form (K3 waits for the other ranks and combines, no K4) applies */
/* Precision of the two operands the default kernel narrows to bf16 where the reference keeps
 * fp32 (reference_decode.py:250-253). Default kernel only (refused with MLA_FLAG_CHECK_KERNEL
 * or MLA_FLAG_TCGEN05). Each costs tensor-core issue in K2, not HBM bytes. */
#define MLA_FLAG_QC_HILO 0x20  /* the absorbed query q_c = q_nope W_UK as a bf16 hi/lo pair: K1 writes both halves,
                                  K2 runs the score MMAs of the 512 latent columns on both (about 16 mantissa bits
                                  of the fp32 q_c instead of 8); the workspace grows by batch x 16 KB */
#define MLA_FLAG_P_HILO 0x40   /* the probabilities of P c_kv as a bf16 hi/lo pair (two MMAs per step) and the row
                                  sums over the unrounded fp32 values, instead of bf16-rounded probabilities */

typedef struct MlaDecodeParams {
    uint32_t struct_size; /* sizeof(MlaDecodeParams) */
    uint32_t abi_version; /* MLA_ABI_VERSION */

    /* dims: must equal the MLA_* constants above */
    int32_t heads, qk_nope, qk_rope, v_head, kv_lora, page_size;
    float softmax_scale; /* q_head_dim^-0.5 * mscale^2 (reference_decode.py:197-203) */
    float rms_eps;       /* kv_a_layernorm eps (1e-6) */

    int32_t batch;      /* requests in this call, 1..MLA_MAX_BATCH */
    int32_t max_blocks; /* row stride of block_table */
    int32_t n_pages;    /* pages in kv_cache */
    int32_t max_pos;    /* rows of rope_cos / rope_sin */

    const void* q;        int64_t q_stride;    /* elements between rows */
    const void* kv_a;     int64_t kv_a_stride; /* elements between rows */
    const void* kv_a_norm_w;
    const void* kv_b;
    const float* rope_cos;
    const float* rope_sin;
    const int32_t* block_table;
    const int32_t* seq_lens;
    void* kv_cache;
    void* out;            int64_t out_stride;  /* elements between rows */

    void* workspace;          /* device scratch, >= mla_workspace_size() bytes, 256-byte aligned */
    uint64_t workspace_bytes;
    int32_t* error_word;      /* optional device int32 (0 = no error); may be NULL */
    int32_t num_ctas;         /* CTAs of the split plan; 0 = the default: two per SM (the default
                                 kernel runs two plan CTAs per CTA), one per SM with MLA_FLAG_TCGEN05 */
    int32_t flags;            /* MLA_FLAG_* */

    /* Sequence-sharded decode (one long sequence split over GPUs by KV range). */
    const int32_t* rope_pos;  /* optional [batch]: RoPE position of the new token (the global position);
                                 NULL = seq_lens[b] */
    float* shard_out;         /* optional: if set, K3 writes this shard's partial instead of `out`:
                                 f32 [batch][16][MLA_SHARD_STRIDE] = y[128] (W_UV o_c / L, normalised
                                 within the shard), m (log2-domain max), L (sum of exps), 2 unused;
                                 16-byte aligned */

    /* In-library q | kv_a projection (ABI v3). If x_n is set, the step first
     * computes q = R(W_q x_n) and kv_a = R(W_kv_a x_n) itself (K0, into the
     * workspace) and q / kv_a above must be NULL. Up to MLA_MAX_PROJECT_BATCH
     * requests K0 streams the weight (m16n8k16); beyond, it is a tcgen05 GEMM (128
     * requests x 64 weight rows x all of K per CTA, accumulators in tensor memory).
     * NULL = q / kv_a are given (ABI v2 behaviour). */
    const void* x_n;          /* [batch][x_stride] bf16 post-RMSNorm hidden state, 16-byte aligned */
    int64_t x_stride;         /* elements between rows, a multiple of 8, >= MLA_HIDDEN */
    const void* w_qkv;        /* [MLA_QKV_ROWS][MLA_HIDDEN] bf16 = rows of q_proj then kv_a_proj_with_mqa,
                                 16-byte aligned */

    /* In-library o_proj with the layer's residual add (ABI v4). If w_o is set,
     * the step ends with h_out = R(residual + R(W_o R(out))) (K5;
     * reference_decode.py:256, 300), reading `out` back (then 16-byte aligned,
     * out_stride a multiple of 8, not with shard_out); the two forms of K0 by
     * batch. NULL = the step ends at R(out). */
    const void* w_o;          /* [MLA_HIDDEN][MLA_HEADS*MLA_V_HEAD] bf16 o_proj.weight, 16-byte aligned */
    const void* residual;     /* [batch][residual_stride] bf16: the layer's input hidden state */
    int64_t residual_stride;  /* elements between rows, a multiple of 4, >= MLA_HIDDEN */
    void* h_out;              /* [batch][h_out_stride] bf16: the new hidden state; may be `residual` itself */
    int64_t h_out_stride;     /* elements between rows, a multiple of 4, >= MLA_HIDDEN */

    /* Sequence-sharded step with the shard exchange over peer memory (ABI v5).
     * world > 0 turns it on. K3 then stores this shard's partial (y, m, L as in
     * shard_out) into slot `rank` of every rank's exchange buffer, with plain stores
     * over NVLink to the peers' memory, each value tagged with the step number in
     * the same 64-bit store; a last kernel (K4) waits until the values of all
     * `world` shards carry this step, bounded by exchange_timeout_us, and combines
     * them in rank order into `out` with the arithmetic of mla_combine_shards. No
     * flag, fence or collective library call is on the path. Where the whole K3
     * grid can be resident at once (small batches), mla_decode_step runs the
     * fused form instead: each K3 CTA waits for the other ranks' values of its own
     * slice and writes `out` itself, with the same arithmetic, and no K4 runs
     * (MLA_FLAG_EXCHANGE_SPLIT keeps K3 + K4).
     * shard_out must be NULL; w_o (K5) may follow. Every rank must run the same
     * sequence of steps with the same batch. world = 0: no exchange. */
    void* exchange[MLA_MAX_RANKS]; /* every rank's exchange buffer as mapped in this process
                                      (mla_exchange_alloc / mla_exchange_open); [rank] is this rank's own */
    int32_t rank;                  /* this shard's index in sequence order, 0..world-1 */
    int32_t world;                 /* number of shards: 0 (no exchange) or 1..MLA_MAX_RANKS */
    int32_t exchange_batch;        /* the batch the buffers were sized for; batch <= exchange_batch */
    int32_t exchange_timeout_us;   /* K4's limit on waiting for a shard; 0 = 2,000,000 (2 s) */

    /* Host-visible device errors (ABI v6). Optional pinned host int32 (cudaHostAlloc /
     * cudaMallocHost memory, which unified addressing maps into the device) that a
     * kernel stores the device error code into whenever it records one in error_word,
     * by a plain store over the system bus. The host can then read it at any time
     * without synchronising with the stream (a kernel's store is visible once that
     * kernel has completed): a caller that checks it before each step learns of a
     * failed step without a device synchronisation, and inside CUDA graphs too. The
     * library never clears it. NULL = no host word. Any other memory is refused with
     * MLA_E_INVALID_ARG. The reference's host polls its abort word the same way
     * (fleet_runtime.h:194-198, read back by fleet_launch.hip:284-311). */
    int32_t* error_host;
} MlaDecodeParams;

#define MLA_SHARD_STRIDE (MLA_V_HEAD + 4)

#define MLA_MAX_BATCH 65536

/* ABI version of the loaded library (MLA_ABI_VERSION). */
int mla_abi_version(void);

/* Human-readable name of an mla_status / device error code. */
const char* mla_status_string(int status);
const char* mla_device_error_string(int code);

/* Fill a params struct with the fixed dims, scale 0 and no pointers. */
void mla_params_init(MlaDecodeParams* p);

/* Bytes of workspace a call with these params needs (depends on batch,
 * num_ctas, the kernel flags and whether x_n is set). Replaces the reference's host-side buffer plan
 * (fleet_types.h:75-81 Activations.q_absorbed/attn_partial; dev_alloc in
 * fleet_launch.hip:223-237): the caller allocates, the library never does. */
int mla_workspace_size(const MlaDecodeParams* p, uint64_t* bytes);

/* Whole attention task: K1 (kv_post + q RoPE + W_UK absorb + split plan),
 * K2 (split-KV attention) and K3 (LSE merge + W_UV), stream-ordered on
 * `stream` (a cudaStream_t; NULL = legacy default stream).
 * Replaces TASK_Q_ABSORB + TASK_ATTENTION + TASK_MERGE_UV as run by
 * fleet_launch_step (fleet_kernel.hip:647-654, :745-798, :694-701, :1068-1078). */
int mla_decode_step(const MlaDecodeParams* p, void* stream);

/* The stages one by one (same params; each expects the previous one's
 * workspace contents). K0 = the q | kv_a projection of x_n (needs p->x_n;
 * reference_decode.py:225-231, device task TASK_QKV_FUSED fleet_kernel.hip:706-741);
 * K1 = kv_post (attention.h:62-90) + q_absorb (attention.h:171-216);
 * K2 = attention_chunk (attention.h:230-351); K3 = merge_and_uv (attention.h:358-411).
 * With p->x_n set, mla_decode_step runs K0 first. */
int mla_project(const MlaDecodeParams* p, void* stream);
int mla_prologue(const MlaDecodeParams* p, void* stream);
/* K5 = o_proj + residual (needs p->w_o; TASK_O_PROJ with the EPI_RESIDUAL
 * epilogue, fleet_kernel.hip:805-824, gemv.h:225). With p->w_o set,
 * mla_decode_step runs it last. */
int mla_o_proj(const MlaDecodeParams* p, void* stream);
int mla_attention(const MlaDecodeParams* p, void* stream);
int mla_merge_uv(const MlaDecodeParams* p, void* stream);

/* Split plan as used by the last K2/K3 of these params, for inspection:
 * number of CTAs that get work and number of partial slots. Host only. */
int mla_plan_info(const MlaDecodeParams* p, int32_t* num_ctas, int32_t* num_slots);

/* Number of kernel launches one mla_decode_step makes (for launch accounting). */
int mla_launches_per_step(void);

/* Combine the shard partials of a sequence-sharded step after they were
 * gathered from all GPUs: parts f32 [n_shards][batch][16][MLA_SHARD_STRIDE]
 * (shard order = sequence order). out[b][128h + v] = bf16(sum_r w_r y_r[v] /
 * sum_r w_r), w_r = L_r * 2^(m_r - max_r m_r), in shard order. The same LSE
 * merge the reference runs over its KV chunks (src/kernels/attention.h:358-401),
 * one level up; there the chunks never leave one GPU. */
int mla_combine_shards(const float* parts, int32_t n_shards, int32_t batch, void* out, int64_t out_stride,
                       void* stream);

/* Exchange buffers of the peer-memory shard exchange (MlaDecodeParams.world > 0).
 * One buffer per rank, allocated by that rank's process on its GPU, zeroed, and
 * mapped into every other rank's process through its CUDA IPC handle; all ranks
 * must use the same world and max_batch. Layout: a step counter and two parities
 * (step & 1) of [world][max_batch][16 heads][65] 16-byte lines; line j < 64 holds
 * y[2j], y[2j+1] and line 64 holds m, L, each as (step << 32) | f32 bits in 64 bits.
 * The reference runs on one GPU and has no counterpart; the exchange replaces an
 * all-gather of the shard partials over a collective library. */
int mla_exchange_bytes(int32_t world, int32_t max_batch, uint64_t* bytes);
/* cudaMalloc + zero on the current device; ipc_handle (MLA_IPC_HANDLE_BYTES, may be
 * NULL) receives the handle that other processes pass to mla_exchange_open. */
int mla_exchange_alloc(uint64_t bytes, void** buf, void* ipc_handle);
int mla_exchange_free(void* buf);
/* Map another process's exchange buffer (peer access enabled lazily). */
int mla_exchange_open(const void* ipc_handle, void** buf);
int mla_exchange_close(void* buf);
/* K4 alone: wait for every shard's flags and combine (needs p->world > 0). In
 * exchange mode mla_merge_uv (K3) must be followed by this call before the next
 * step; mla_decode_step runs both. */
int mla_exchange_combine(const MlaDecodeParams* p, void* stream);

/* Prefill hand-off: rows of a prefill into the paged cache. Replaces the
 * reference's flat per-layer cache [max_pos][576] bf16, built from the hooked
 * kv_a_proj_with_mqa output by src/host/kv_convert.py:36-139 and uploaded as-is
 * by src/host/fleet_launch.hip:651-669; here each request's rows are scattered
 * into its pages at positions first_pos[b], first_pos[b] + 1, ... */
#define MLA_ROWS_FINAL 0  /* rows are cache rows already (c after kv_a_layernorm | k_pe after RoPE): copied;
                             this is the reference's cache-file row format */
#define MLA_ROWS_RAW 1    /* rows are raw kv_a (the kv_a_proj_with_mqa output): kv_a_layernorm and RoPE at the
                             row's position are applied, with the arithmetic of the decode step's new row */

typedef struct MlaRowsToPages {
    uint32_t struct_size;      /* sizeof(MlaRowsToPages) */
    uint32_t abi_version;      /* MLA_ABI_VERSION */
    int32_t mode;              /* MLA_ROWS_FINAL or MLA_ROWS_RAW */
    int32_t batch;             /* requests, 1..MLA_MAX_BATCH */
    int64_t total_rows;        /* row_start[batch], as known to the host (sizes the grid) */
    const void* rows;          /* bf16 [total_rows][rows_stride], 16-byte aligned */
    int64_t rows_stride;       /* elements between rows: >= 576, a multiple of 8 */
    const int64_t* row_start;  /* device [batch + 1]: request b's rows are rows[row_start[b], row_start[b+1]) */
    const int32_t* first_pos;  /* device [batch]: position of request b's first row; NULL = 0 */
    const int32_t* block_table;
    int32_t max_blocks;
    int32_t n_pages;
    void* kv_cache;            /* [n_pages][64][576] bf16, 16-byte aligned */
    const void* kv_a_norm_w;   /* MLA_ROWS_RAW: bf16 [512] kv_a_layernorm.weight */
    const float* rope_cos;     /* MLA_ROWS_RAW: [max_pos][64] YaRN tables */
    const float* rope_sin;
    int32_t max_pos;           /* MLA_ROWS_RAW */
    float rms_eps;             /* MLA_ROWS_RAW */
    int32_t* error_word;       /* optional: MLA_DEV_BAD_POSITION / MLA_DEV_BAD_PAGE; such rows are skipped */
} MlaRowsToPages;

/* Fill an MlaRowsToPages with its size and version, everything else zero. */
void mla_rows_init(MlaRowsToPages* r);

int mla_rows_to_pages(const MlaRowsToPages* r, void* stream);

/* Size of the workspace that mla_decode_step_static keeps inside the library, per
 * device: 32 MiB, which holds mla_workspace_size() for up to 463 requests at the
 * default 296 split-KV CTAs of a B200 (558 at num_ctas = 148). */
#define MLA_STATIC_SCRATCH_BYTES (32ull << 20)

/* No counterpart in the reference: its launcher allocates every buffer itself
 * before the token loop (fleet_launch.hip:223-237), so it never needed this.
 *
 * mla_decode_step with the workspace taken from a device array inside the library
 * (MLA_STATIC_SCRATCH_BYTES per device) instead of from the caller. p->workspace
 * and p->workspace_bytes are ignored; every other field means what it means for
 * mla_decode_step, and the same kernels run. It calls no cudaMalloc, cudaFree or
 * other allocating routine. It is for callers that cannot allocate device memory
 * on the decode path: a server that sized its paged KV pool to all the HBM left
 * after the weights has none left for a per-step workspace, and a C or FFI host
 * without a caching allocator would otherwise pay a cudaMalloc/cudaFree (and the
 * device-wide synchronisation of cudaFree) per decoded token whenever the batch grows.
 *
 * Returns MLA_E_LIMIT, before any launch, when mla_workspace_size(p) exceeds
 * MLA_STATIC_SCRATCH_BYTES. Nothing in the scratch has to start at zero (each
 * step writes everything it reads). The scratch is one per device and shared by
 * every call on that device: calls that overlap on the GPU (on streams not
 * ordered with one another, or from several host threads) race on it. Order
 * them on one stream or with events. The first call on a device, with that device
 * current, looks up the scratch array's device address (cudaGetSymbolAddress);
 * make that first call before any stream capture on that device. A lookup that
 * fails returns MLA_E_LAUNCH and is not remembered: the next call tries again. */
int mla_decode_step_static(const MlaDecodeParams* p, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* MLA_DECODE_H_ */
