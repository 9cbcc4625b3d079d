// mla_decode_step_static: the decode step with its workspace in a device array
// of this library instead of in caller memory, for callers that cannot allocate
// on the decode path (declared in include/mla_decode.h, which says who they are).
//
// The three kernels and their checks are those of mla_decode_step; only the
// workspace pointer differs. Nothing is allocated: the array is part of this
// file's device image, and its address is looked up once per device.
#include <atomic>
#include <mutex>

#include "mla_common.cuh"

namespace {

// One per device. Nothing in it has to start at zero: in every step K1 writes
// the tile plan and the absorbed queries before K2 reads them, K2 writes every
// partial slot that K3 reads, and K3 reads nothing else. Calls that overlap on
// the GPU share this one array and race on it.
static __device__ __align__(256) unsigned char g_static_scratch[MLA_STATIC_SCRATCH_BYTES];

constexpr int kMaxDevices = 64;

struct ScratchSlot {
    std::mutex mu;                    // serialises the lookup
    std::atomic<void*> ptr{nullptr};  // set once a lookup has succeeded; a failed one is retried
};
ScratchSlot g_slots[kMaxDevices];

// Device address of g_static_scratch on the current device, looked up at the
// first call on that device (with that device current). Only a successful
// lookup is kept, so a first call that failed (made during a stream capture,
// say) does not disable the entry point: the next call looks it up again.
int static_scratch(void** ptr) {
    int dev = -1;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return MLA_E_LAUNCH;
    ScratchSlot& s = g_slots[dev];
    void* p = s.ptr.load(std::memory_order_acquire);
    if (!p) {
        std::lock_guard<std::mutex> lock(s.mu);
        p = s.ptr.load(std::memory_order_relaxed);
        if (!p) {
            if (cudaGetSymbolAddress(&p, g_static_scratch) != cudaSuccess || p == nullptr) {
                cudaGetLastError();  // leave no error behind for the caller's next CUDA call
                return MLA_E_LAUNCH;
            }
            s.ptr.store(p, std::memory_order_release);
        }
    }
    *ptr = p;
    return MLA_OK;
}

}  // namespace

extern "C" int mla_decode_step_static(const MlaDecodeParams* p, void* stream) {
    uint64_t need = 0;
    int st = mla_workspace_size(p, &need);  // header, dims, batch and CTA-count checks
    if (st != MLA_OK) return st;
    if (need > MLA_STATIC_SCRATCH_BYTES) return MLA_E_LIMIT;
    void* scratch = nullptr;
    st = static_scratch(&scratch);
    if (st != MLA_OK) return st;
    MlaDecodeParams q = *p;
    q.workspace = scratch;
    q.workspace_bytes = MLA_STATIC_SCRATCH_BYTES;
    return mla_decode_step(&q, stream);
}
