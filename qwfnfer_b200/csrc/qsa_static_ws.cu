// qsa_static_ws.cu -- qsa_decode for callers that cannot allocate device memory.
//
// Some callers of the decode node cannot hand the library a workspace: an operator invoked from
// inside another framework's graph executor only sees the tensors that executor planned (its
// buffers are laid out before the graph runs, so nothing can be allocated in the middle of it),
// and a serving loop that runs under a fixed memory budget must not call cudaMalloc on the
// token path (it synchronises the device and can fail under fragmentation).  For them the
// scratch of one decode call lives in a fixed, file-scope device array instead.
#include <mutex>

#include "qsa_kernels.cuh"

namespace {

// Maximum scratch of one call.  Every GPU that loads the library holds this array until exit.
constexpr size_t QSA_STATIC_SCRATCH_BYTES = 8u << 20;   // 8 MiB

static __device__ __align__(256) unsigned char g_qsa_static_scratch[QSA_STATIC_SCRATCH_BYTES];

constexpr int MAX_DEVICES = 64;
std::mutex g_setup_mu;
void * g_scratch_addr[MAX_DEVICES];   // the array's device address, per device (set up on first use)

// Device address of the array on the current device.  In host code the array's name is only a
// host-side stand-in; the address kernels may use comes from cudaGetSymbolAddress, taken once
// per device with that device current.  Nothing is written here: each call zeroes the part of
// the array that must start at zero on the caller's stream (a memset on another stream would be
// unordered against a non-blocking caller stream).
qsa_status scratch_for_current_device(void ** out) {
    int dev = -1;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= MAX_DEVICES) return QSA_ERR_CUDA;
    std::lock_guard<std::mutex> lock(g_setup_mu);
    if (!g_scratch_addr[dev]) {
        void * p = nullptr;
        if (cudaGetSymbolAddress(&p, g_qsa_static_scratch) != cudaSuccess || !p) return QSA_ERR_CUDA;
        g_scratch_addr[dev] = p;
    }
    *out = g_scratch_addr[dev];
    return QSA_OK;
}

}  // namespace

extern "C" qsa_status qsa_decode_noalloc(const qsa_desc * d, const qsa_decode_item * items, int32_t batch,
                                         int32_t max_n_kv, const void * q, int32_t q_type, const float * q_idx,
                                         const float * k_new, const float * v_new, const float * kidx_new,
                                         float * out, int32_t * sel_out, qsa_stream_t stream) {
    qsa_status s = qsa_desc_check(d);
    if (s != QSA_OK) return s;
    const size_t need = qsa_decode_workspace_size(d, batch, max_n_kv);
    if (need == 0) return QSA_ERR_INVALID;
    if (need > QSA_STATIC_SCRATCH_BYTES) return QSA_ERR_WORKSPACE;      // beyond the fixed maximum
    void * ws = nullptr;
    if ((s = scratch_for_current_device(&ws)) != QSA_OK) return s;
    // The array keeps the previous call's contents, and the workspace layout moves with the batch
    // size: zero the status word and arrival counters (the layout's leading region, the only part
    // the kernels read before writing) every call, on the caller's stream.
    const size_t zero_bytes = qsa::decode_workspace_zero_prefix(d, batch, max_n_kv);
    if (cudaMemsetAsync(ws, 0, zero_bytes, reinterpret_cast<cudaStream_t>(stream)) != cudaSuccess) return QSA_ERR_CUDA;
    return qsa_decode(d, items, batch, max_n_kv, q, q_type, q_idx, k_new, v_new, kidx_new, out, sel_out,
                      ws, need, stream);
}
