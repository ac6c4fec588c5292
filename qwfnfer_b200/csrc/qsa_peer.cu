// qsa_peer.cu -- all-gather of small per-rank slices over NVLink peer memory, for the exchanges
// of the KV-sequence-sharded decode (candidates, attention states).
//
// Each rank owns one gather buffer: n_ranks slots of slot_bytes (a multiple of 4) at a stride
// rounded up to 16 bytes, followed by n_ranks uint32 flags.
// Every rank maps the buffers of all ranks (CUDA IPC; plain peer loads/stores over NVLink).
//   qsa_peer_push: copy this rank's slice into slot `rank` of every rank's buffer with peer
//     stores, then, after a system-scope fence, set flag[rank] = epoch in every buffer.  The epoch
//     is a per-rank device counter that push increments (every rank pushes the same number of
//     times, so the values agree).
//   qsa_peer_wait: spin (bounded: 2 s of %globaltimer, then DEV_TIMEOUT in the status word) until
//     every flag of this rank's buffer carries the current epoch; kernels launched after it read
//     the gathered slots.
//   qsa_shard_decode_ri_peer's publication (peer_publish_kernel): the attention (or its merge)
//     has stored this rank's states into slot `rank` of every buffer itself; once that grid has
//     completed, one warp advances the epoch and sets flag[rank] in every buffer with a
//     system-scope release, and qsa_merge_states_peer waits for the flags.
// No multicast and no NVLS: only ordinary stores to peer memory and loads of local memory.
#include <cstring>

#include "qsa_kernels.cuh"

namespace qsa {

constexpr int PEER_THREADS = 256;

__device__ __forceinline__ void st_release_sys(uint32_t * p, uint32_t v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" :: "l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t * p) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__host__ __device__ __forceinline__ size_t peer_stride(size_t slot_bytes) { return (slot_bytes + 15) & ~(size_t) 15; }

// grid = CTAs, each copying its share of the slice to every rank (a few KB per rank, so usually one
// CTA).  Every CTA fences its peer stores at system scope before it counts itself; the last CTA
// to finish publishes the flags.
__global__ void __launch_bounds__(PEER_THREADS) peer_push_kernel(void * const * __restrict__ bufs, int n_ranks, int rank,
        const void * __restrict__ src, size_t slot_bytes, uint32_t * __restrict__ epoch, unsigned * __restrict__ counter) {
    __shared__ bool last;
    const size_t stride = peer_stride(slot_bytes);
    const size_t n16 = slot_bytes / 16;
    const uint4 * s4 = static_cast<const uint4 *>(src);
    for (size_t i = (size_t) blockIdx.x * PEER_THREADS + threadIdx.x; i < n16; i += (size_t) gridDim.x * PEER_THREADS) {
        const uint4 v = s4[i];
        for (int p = 0; p < n_ranks; p++)
            reinterpret_cast<uint4 *>(static_cast<unsigned char *>(bufs[p]) + (size_t) rank * stride)[i] = v;
    }
    if (blockIdx.x == 0 && threadIdx.x < (slot_bytes % 16) / 4) {    // the 4-byte tail
        const uint32_t v = reinterpret_cast<const uint32_t *>(static_cast<const unsigned char *>(src) + n16 * 16)[threadIdx.x];
        for (int p = 0; p < n_ranks; p++)
            reinterpret_cast<uint32_t *>(static_cast<unsigned char *>(bufs[p]) + (size_t) rank * stride + n16 * 16)[threadIdx.x] = v;
    }
    __threadfence_system();                  // this CTA's peer stores are visible before any flag
    __syncthreads();
    if (threadIdx.x == 0) {
        unsigned prev;
        asm volatile("atom.add.acq_rel.gpu.u32 %0, [%1], 1;" : "=r"(prev) : "l"(counter) : "memory");
        last = prev == gridDim.x - 1;
    }
    __syncthreads();
    if (!last) return;
    if (threadIdx.x == 0) {
        *counter = 0;
        *epoch = *epoch + 1;
    }
    __syncthreads();
    const uint32_t e = *reinterpret_cast<volatile uint32_t *>(epoch);
    if ((int) threadIdx.x < n_ranks) {
        uint32_t * flags = reinterpret_cast<uint32_t *>(static_cast<unsigned char *>(bufs[threadIdx.x]) + (size_t) n_ranks * stride);
        st_release_sys(flags + rank, e);
    }
}

__global__ void peer_wait_kernel(const void * __restrict__ local_buf, int n_ranks, size_t slot_bytes,
                                 const uint32_t * __restrict__ epoch, uint32_t * __restrict__ status) {
    const int r = threadIdx.x;
    if (r >= n_ranks) return;
    const uint32_t * flags = reinterpret_cast<const uint32_t *>(static_cast<const unsigned char *>(local_buf) +
                                                                (size_t) n_ranks * peer_stride(slot_bytes));
    // A flag at or past this round's epoch means the peer's slice of this round has landed (the
    // difference as a signed value, so the test survives the counter wrapping).
    const uint32_t e = *epoch;
    if ((int32_t) (ld_acquire_sys(flags + r) - e) < 0) {
        const uint64_t t0 = global_timer_ns();
        while ((int32_t) (ld_acquire_sys(flags + r) - e) < 0) {
            if (global_timer_ns() - t0 > 2000000000ull) {
                set_status(status, DEV_TIMEOUT);
                break;
            }
        }
    }
    __threadfence_system();
}

// Publication of states that the kernel ahead stored into every rank's region (StateDst with the
// regions' slots of this rank): once that grid has completed (its stores performed), the channel's
// next epoch goes into this rank's flag of every region with a system-scope release.
struct PeerFlags {
    uint32_t * flag[MAX_STATE_DST];
};
__global__ void peer_publish_kernel(PeerFlags f, int n, uint32_t * __restrict__ epoch) {
    pdl_wait();                              // the grid that stored the states has completed
    __shared__ uint32_t e;
    if (threadIdx.x == 0) {
        e = *epoch + 1;
        *epoch = e;
    }
    __syncthreads();
    if ((int) threadIdx.x < n) {
        __threadfence_system();
        st_release_sys(f.flag[threadIdx.x], e);
    }
}

cudaError_t launch_peer_publish(cudaStream_t st, uint32_t * const * flag, int n, uint32_t * epoch) {
    if (n <= 0 || n > MAX_STATE_DST) return cudaErrorInvalidValue;
    PeerFlags f{};
    for (int p = 0; p < n; p++) f.flag[p] = flag[p];
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(1);
    cfg.blockDim = dim3(32);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;      // its launch overlaps the writer
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, peer_publish_kernel, f, n, epoch);
}

cudaError_t launch_peer_push(cudaStream_t st, void * const * bufs, int n_ranks, int rank, const void * src,
                             size_t slot_bytes, uint32_t * epoch, unsigned * counter) {
    // about 32 KB of peer stores per CTA
    const int ctas = (int) std::min<size_t>(32, std::max<size_t>(1, (slot_bytes * n_ranks + 32767) / 32768));
    peer_push_kernel<<<ctas, PEER_THREADS, 0, st>>>(bufs, n_ranks, rank, src, slot_bytes, epoch, counter);
    return cudaGetLastError();
}

cudaError_t launch_peer_wait(cudaStream_t st, const void * local_buf, int n_ranks, size_t slot_bytes,
                             const uint32_t * epoch, uint32_t * status) {
    peer_wait_kernel<<<1, 32, 0, st>>>(local_buf, n_ranks, slot_bytes, epoch, status);
    return cudaGetLastError();
}

}  // namespace qsa

using namespace qsa;

namespace {
// Base and size of the allocation holding a device pointer: the driver's cuMemGetAddressRange,
// reached through the runtime's entry-point query (no link-time dependency on the driver library).
cudaError_t allocation_base(const void * ptr, void ** base) {
    typedef int (*range_fn)(unsigned long long *, size_t *, unsigned long long);
    static range_fn fn = nullptr;
    if (!fn) {
        void * f = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &f, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess || !f)
            return cudaErrorNotSupported;
        fn = reinterpret_cast<range_fn>(f);
    }
    unsigned long long b = 0;
    size_t size = 0;
    if (fn(&b, &size, (unsigned long long) reinterpret_cast<uintptr_t>(ptr)) != 0) return cudaErrorInvalidValue;
    *base = reinterpret_cast<void *>((uintptr_t) b);
    return cudaSuccess;
}
}  // namespace

extern "C" {

qsa_status qsa_ipc_handle(const void * ptr, void * handle, size_t * offset) {
    if (!ptr || !handle || !offset) return QSA_ERR_INVALID;
    void * base = nullptr;
    if (allocation_base(ptr, &base) != cudaSuccess) return QSA_ERR_CUDA;
    cudaIpcMemHandle_t h;
    if (cudaIpcGetMemHandle(&h, base) != cudaSuccess) return QSA_ERR_CUDA;
    std::memcpy(handle, &h, sizeof h);
    *offset = (size_t) (static_cast<const unsigned char *>(ptr) - static_cast<unsigned char *>(base));
    return QSA_OK;
}

qsa_status qsa_ipc_open(const void * handle, void ** base) {
    if (!handle || !base) return QSA_ERR_INVALID;
    cudaIpcMemHandle_t h;
    std::memcpy(&h, handle, sizeof h);
    return cudaIpcOpenMemHandle(base, h, cudaIpcMemLazyEnablePeerAccess) == cudaSuccess ? QSA_OK : QSA_ERR_CUDA;
}

qsa_status qsa_ipc_close(void * base) {
    return cudaIpcCloseMemHandle(base) == cudaSuccess ? QSA_OK : QSA_ERR_CUDA;
}

size_t qsa_peer_buffer_bytes(int32_t n_ranks, size_t slot_bytes) {
    if (n_ranks <= 0 || n_ranks > 32 || slot_bytes == 0 || slot_bytes % 4 != 0) return 0;
    return (size_t) n_ranks * peer_stride(slot_bytes) + (size_t) ((n_ranks * 4 + 255) & ~255);
}

qsa_status qsa_peer_push(void * const * bufs, int32_t n_ranks, int32_t rank, const void * src, size_t slot_bytes,
                         uint32_t * epoch, uint32_t * counter, qsa_stream_t stream) {
    if (!bufs || !src || !epoch || !counter || n_ranks <= 0 || n_ranks > 32 || rank < 0 || rank >= n_ranks ||
        slot_bytes == 0 ||
        slot_bytes % 4 != 0 || reinterpret_cast<uintptr_t>(src) % 16 != 0)
        return QSA_ERR_INVALID;
    return launch_peer_push(reinterpret_cast<cudaStream_t>(stream), bufs, n_ranks, rank, src, slot_bytes, epoch,
                            counter) == cudaSuccess ? QSA_OK : QSA_ERR_CUDA;
}

qsa_status qsa_peer_wait(const void * local_buf, int32_t n_ranks, size_t slot_bytes, const uint32_t * epoch,
                         void * ws, size_t ws_bytes, qsa_stream_t stream) {
    if (!local_buf || !epoch || n_ranks <= 0 || n_ranks > 32 || slot_bytes == 0 || slot_bytes % 4 != 0)
        return QSA_ERR_INVALID;
    if (!ws || ws_bytes < 16) return QSA_ERR_WORKSPACE;
    return launch_peer_wait(reinterpret_cast<cudaStream_t>(stream), local_buf, n_ranks, slot_bytes, epoch,
                            static_cast<uint32_t *>(ws)) == cudaSuccess ? QSA_OK : QSA_ERR_CUDA;
}

}  // extern "C"
