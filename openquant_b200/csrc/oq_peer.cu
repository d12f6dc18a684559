// Peer memory of the N-column-sharded linear layer: one process per GPU,
// each GPU's output buffer mapped into every other GPU of the node (CUDA IPC
// over NVLink / NVSwitch -- plain peer mappings, no multicast objects), and
// a flag barrier that tells each GPU when all of its peers' stores into its
// buffer have landed.
//
// The sharded layer's kernels (oq_int4_linear_peers) store every output
// element of their slice into all GPUs' buffers; oq_peer_barrier, enqueued
// after them on the same stream, then
//   1. counts itself (epoch = this GPU's barrier count, kept in its own flag
//      array), orders everything the stream's earlier kernels wrote (the peer
//      stores included) before a release store of `epoch` into slot `rank` of
//      every GPU's flag array, and
//   2. waits, with acquire loads bounded by a timeout, until every slot of
//      its own flag array holds `epoch` or later -- i.e. every GPU has
//      finished its stores into this GPU's buffer.
// A wait that runs out records OQ_DEV_PEER_TIMEOUT in the device error word
// (oq_take_device_error) and returns; nothing waits forever.
#include "oq_sm100.cuh"

#include <cstring>

namespace oq {
namespace {

constexpr int OQ_DEV_PEER_TIMEOUT = 2;
constexpr long long kDefaultPeerTimeoutNs = 5ll * 1000 * 1000 * 1000;

struct FlagPtrs {
    uint32_t *gpu[kMaxOutGpus];
};

__device__ __forceinline__ uint64_t global_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ void st_release_sys(uint32_t *p, uint32_t v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t *p) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__global__ void __launch_bounds__(32) peer_barrier_kernel(FlagPtrs flags, int world, int rank, long long timeout_ns) {
    __shared__ uint32_t epoch_s;
    const int t = threadIdx.x;
    uint32_t *own = flags.gpu[rank];
    // This GPU's barrier count: only this kernel touches it, and launches on
    // one stream run one after another, so a plain update is enough.  Kept on
    // the device so that a CUDA graph of the layer replays correctly.
    if (t == 0) {
        const uint32_t e = own[OQ_PEER_FLAG_WORDS - 1] + 1;
        own[OQ_PEER_FLAG_WORDS - 1] = e;
        epoch_s = e;
    }
    __syncthreads();
    const uint32_t epoch = epoch_s;
    if (t >= world) return;
    // The stream's earlier kernels have completed before this grid started;
    // the system-scope fence and release store publish their writes (on this
    // GPU and the peer stores alike) to GPU t before it can see the flag.
    __threadfence_system();
    st_release_sys(flags.gpu[t] + rank, epoch);
    const uint32_t *mine = own + t;
    const uint64_t t0 = global_ns();
    while ((int32_t)(ld_acquire_sys(mine) - epoch) < 0) {
        if ((long long)(global_ns() - t0) > timeout_ns || *(volatile int *)&g_device_error != 0) {
            record_device_error(OQ_DEV_PEER_TIMEOUT);
            return;
        }
        __nanosleep(64);
    }
}

}  // namespace
}  // namespace oq

using namespace oq;

extern "C" int oq_peer_alloc(size_t bytes, void **ptr) {
    clear_error();
    OQ_REQUIRE(ptr != nullptr && bytes > 0, "peer buffer: need a size and an output pointer");
    *ptr = nullptr;
    void *p = nullptr;
    OQ_CUDA(cudaMalloc(&p, bytes));
    cudaError_t e = cudaMemset(p, 0, bytes);
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    if (e != cudaSuccess) {
        cudaFree(p);
        set_error("peer buffer: zeroing failed: %s", cudaGetErrorString(e));
        return OQ_ERR_CUDA;
    }
    *ptr = p;
    return OQ_OK;
}

extern "C" int oq_peer_free(void *ptr) {
    clear_error();
    if (ptr == nullptr) return OQ_OK;
    OQ_CUDA(cudaFree(ptr));
    return OQ_OK;
}

extern "C" int oq_peer_export(const void *ptr, uint8_t *handle) {
    clear_error();
    static_assert(sizeof(cudaIpcMemHandle_t) == OQ_PEER_HANDLE_BYTES, "IPC handle size");
    OQ_REQUIRE(ptr != nullptr && handle != nullptr, "null pointer argument");
    cudaIpcMemHandle_t h;
    OQ_CUDA(cudaIpcGetMemHandle(&h, const_cast<void *>(ptr)));
    memcpy(handle, &h, sizeof(h));
    return OQ_OK;
}

extern "C" int oq_peer_import(const uint8_t *handle, void **ptr) {
    clear_error();
    OQ_REQUIRE(ptr != nullptr && handle != nullptr, "null pointer argument");
    *ptr = nullptr;
    cudaIpcMemHandle_t h;
    memcpy(&h, handle, sizeof(h));
    OQ_CUDA(cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess));
    return OQ_OK;
}

extern "C" int oq_peer_close(void *ptr) {
    clear_error();
    if (ptr == nullptr) return OQ_OK;
    OQ_CUDA(cudaIpcCloseMemHandle(ptr));
    return OQ_OK;
}

extern "C" int oq_peer_barrier(uint32_t *const *flags_gpus, int world, int rank, int64_t timeout_ns,
                               oq_stream_t stream) {
    clear_error();
    OQ_REQUIRE(flags_gpus != nullptr && world >= 1 && world <= kMaxOutGpus, "world must be in [1, %d]",
               kMaxOutGpus);
    OQ_REQUIRE(rank >= 0 && rank < world, "rank must be in [0, world)");
    OQ_REQUIRE(timeout_ns >= 0, "timeout must be >= 0");
    FlagPtrs f = {};
    for (int i = 0; i < world; ++i) {
        OQ_REQUIRE(flags_gpus[i] != nullptr && aligned(flags_gpus[i], 4), "flag array %d: null or unaligned", i);
        f.gpu[i] = flags_gpus[i];
    }
    peer_barrier_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(
        f, world, rank, timeout_ns > 0 ? (long long)timeout_ns : kDefaultPeerTimeoutNs);
    return check_launch("peer barrier");
}
