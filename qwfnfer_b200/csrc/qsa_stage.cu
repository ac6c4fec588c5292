// qsa_stage.cu -- host<->device staging of a decode step's activations by a kernel.
//
// A decode step's inputs (the item table, q, q_idx and the new token's K/V/indexer rows: about
// 13 KB at batch 1) and its output (16 KB) are tiny.  Moving them with cudaMemcpyAsync hands
// them to a copy engine, and each hand-over between the copy engine and the compute engine
// costs several microseconds of latency at either end of the step.  A kernel that reads pinned
// host memory (mapped into the device's address space at its host address, as every pinned
// allocation is on a system with unified addressing) moves the same bytes in one PCIe round
// trip and chains to the decode kernels with programmatic dependent launch.  The reference's
// engine sets its per-token decode inputs with ggml_backend_tensor_set (src/qwfn_engine.cpp:738-753)
// before the step's graph is computed (src/qwfn_engine.cpp:814).
#include "qsa_kernels.cuh"

namespace qsa {
namespace {

constexpr int STAGE_THREADS = 256;

// 16-byte pieces, one per thread and grid-stride beyond that.  The wait comes first: the bytes
// may be the output of the kernel before this one in the stream.
__global__ void __launch_bounds__(STAGE_THREADS) stage_copy_kernel(uint4 * __restrict__ dst,
                                                                   const uint4 * src, size_t n16) {
    pdl_wait();
    pdl_trigger();
    const size_t stride = (size_t) gridDim.x * blockDim.x;
    for (size_t i = (size_t) blockIdx.x * blockDim.x + threadIdx.x; i < n16; i += stride) dst[i] = ld_dep(src + i);
}

// Device memory of the current device, managed memory, or pinned host memory that kernels can
// reach at its host address.
bool device_accessible(const void * p) {
    cudaPointerAttributes a{};
    if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
        (void) cudaGetLastError();
        return false;
    }
    int dev = -1;
    if (cudaGetDevice(&dev) != cudaSuccess) return false;
    if (a.type == cudaMemoryTypeDevice) return a.device == dev;
    if (a.type == cudaMemoryTypeManaged) return true;
    return a.type == cudaMemoryTypeHost && a.devicePointer == p;
}

}  // namespace
}  // namespace qsa

using namespace qsa;

extern "C" qsa_status qsa_stage_copy(void * dst, const void * src, size_t bytes, qsa_stream_t stream) {
    if (!dst || !src || bytes == 0 || bytes % 16 != 0) return QSA_ERR_INVALID;
    if (reinterpret_cast<uintptr_t>(dst) % 16 != 0 || reinterpret_cast<uintptr_t>(src) % 16 != 0) return QSA_ERR_INVALID;
    if (!device_accessible(dst) || !device_accessible(src)) return QSA_ERR_INVALID;
    const size_t n16 = bytes / 16;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned) std::min<size_t>((n16 + STAGE_THREADS - 1) / STAGE_THREADS, 4 * 148));
    cfg.blockDim = dim3(STAGE_THREADS);
    cfg.stream = reinterpret_cast<cudaStream_t>(stream);
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaError_t e = cudaLaunchKernelEx(&cfg, stage_copy_kernel, static_cast<uint4 *>(dst),
                                       static_cast<const uint4 *>(src), n16);
    return e == cudaSuccess ? QSA_OK : QSA_ERR_CUDA;
}
