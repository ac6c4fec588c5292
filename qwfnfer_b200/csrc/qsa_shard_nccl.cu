// qsa_shard_nccl.cu -- the whole KV-sequence-sharded decode step behind the C ABI, its two
// exchanges done with the caller's NCCL communicator.
//
// The shard calls of qsa_api.cu (candidates, attend, merge) leave the all-gathers to the caller;
// an engine without a Python layer would re-implement that orchestration.  qsa_decode_sharded does
// it: on every rank, with the same arguments except the shard's block range,
//   sharded indexer caches:    qsa_shard_candidates -> ncclAllGather(candidates) -> qsa_shard_attend
//   replicated indexer caches: qsa_shard_decode_ri (every rank selects globally itself)
// then ncclAllGather(states) -> qsa_merge_states, all on `stream` (capturable in a CUDA graph like
// any NCCL call).  NCCL is not linked: its entry points are taken from the libnccl.so.2 already
// loaded in the process (the one that created the communicator), so the library adds no NCCL
// dependency of its own and never mixes two NCCL builds.
#include <dlfcn.h>

#include <mutex>

#include "qsa_kernels.cuh"

namespace {

// ncclAllGather(sendbuff, recvbuff, sendcount, ncclDataType_t, ncclComm_t, cudaStream_t) and
// ncclCommCount(ncclComm_t, int *); the enum and handle types passed as their ABI types.
typedef int (*nccl_allgather_fn)(const void *, void *, size_t, int, void *, cudaStream_t);
typedef int (*nccl_count_fn)(const void *, int *);
constexpr int NCCL_INT32 = 2, NCCL_FLOAT32 = 7;       // ncclInt32, ncclFloat32

struct NcclApi {
    nccl_allgather_fn allgather = nullptr;
    nccl_count_fn count = nullptr;
};

const NcclApi * nccl_api() {
    static std::once_flag once;
    static NcclApi api;
    std::call_once(once, [] {
        void * h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);      // only an instance already loaded
        if (!h) return;
        api.allgather = reinterpret_cast<nccl_allgather_fn>(dlsym(h, "ncclAllGather"));
        api.count = reinterpret_cast<nccl_count_fn>(dlsym(h, "ncclCommCount"));
    });
    return api.allgather && api.count ? &api : nullptr;
}

size_t a256(size_t x) { return (x + 255) & ~(size_t) 255; }

struct ShardedWs { size_t shard, cand, cand_all, state, state_all, total; };

ShardedWs sharded_ws(const qsa_desc * d, int32_t batch, int32_t max_n_kv, int32_t blk_lo, int32_t blk_hi, int32_t n_ranks) {
    ShardedWs w{};
    const size_t inner = qsa_shard_workspace_size(d, batch, max_n_kv, blk_lo, blk_hi);
    if (!inner) return w;
    const size_t cand = (size_t) 2 * batch * qsa_k_blocks(d) * 4;
    const size_t state = (size_t) batch * qsa_shard_state_floats(d) * 4;
    w.shard = 0;
    w.cand = a256(inner);
    w.cand_all = w.cand + a256(cand);
    w.state = w.cand_all + a256(cand * n_ranks);
    w.state_all = w.state + a256(state);
    w.total = w.state_all + a256(state * n_ranks);
    return w;
}

}  // namespace

extern "C" size_t qsa_decode_sharded_workspace_size(const qsa_desc * d, int32_t batch, int32_t max_n_kv,
                                                    int32_t blk_lo, int32_t blk_hi, int32_t n_ranks) {
    if (n_ranks <= 0) return 0;
    return sharded_ws(d, batch, max_n_kv, blk_lo, blk_hi, n_ranks).total;
}

extern "C" qsa_status qsa_decode_sharded(const qsa_desc * d, const qsa_decode_item * items, int32_t batch,
                                         int32_t max_n_kv, int32_t blk_lo, int32_t blk_hi, int32_t index_replicated,
                                         qsa_nccl_comm_t comm, int32_t n_ranks,
                                         const void * q, int32_t q_type, const float * q_idx,
                                         const float * k_new, const float * v_new, const float * kidx_new,
                                         float * out, int32_t * sel_out, void * ws, size_t ws_bytes,
                                         qsa_stream_t stream) {
    qsa_status s = qsa_desc_check(d);
    if (s != QSA_OK) return s;
    if (!comm || n_ranks <= 0 || !out || batch <= 0) return QSA_ERR_INVALID;
    const NcclApi * nc = nccl_api();
    if (!nc) return QSA_ERR_UNSUPPORTED;                  // no NCCL loaded in this process
    int count = 0;
    if (nc->count(comm, &count) != 0 || count != n_ranks) return QSA_ERR_INVALID;
    const ShardedWs L = sharded_ws(d, batch, max_n_kv, blk_lo, blk_hi, n_ranks);
    if (!L.total) return QSA_ERR_INVALID;
    if (!ws || ws_bytes < L.total) return QSA_ERR_WORKSPACE;
    unsigned char * wsb = static_cast<unsigned char *>(ws);
    const size_t inner = L.cand;                          // the shard calls' workspace, at the start
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    const int kb = qsa_k_blocks(d);
    const size_t sf = qsa_shard_state_floats(d);
    float * state = reinterpret_cast<float *>(wsb + L.state);
    float * state_all = reinterpret_cast<float *>(wsb + L.state_all);
    if (index_replicated) {
        s = qsa_shard_decode_ri(d, items, batch, max_n_kv, blk_lo, blk_hi, q, q_type, q_idx, k_new, v_new, kidx_new,
                                state, sel_out, wsb, inner, stream);
        if (s != QSA_OK) return s;
    } else {
        int32_t * cand = reinterpret_cast<int32_t *>(wsb + L.cand);
        int32_t * cand_all = reinterpret_cast<int32_t *>(wsb + L.cand_all);
        s = qsa_shard_candidates(d, items, batch, max_n_kv, blk_lo, blk_hi, q_idx, k_new, v_new, kidx_new, cand, wsb,
                                 inner, stream);
        if (s != QSA_OK) return s;
        if (nc->allgather(cand, cand_all, (size_t) 2 * batch * kb, NCCL_INT32, comm, st) != 0) return QSA_ERR_CUDA;
        s = qsa_shard_attend(d, items, batch, max_n_kv, blk_lo, blk_hi, n_ranks, cand_all, 0, q, q_type, state, sel_out,
                             wsb, inner, stream);
        if (s != QSA_OK) return s;
    }
    if (nc->allgather(state, state_all, (size_t) batch * sf, NCCL_FLOAT32, comm, st) != 0) return QSA_ERR_CUDA;
    return qsa_merge_states(d, n_ranks, batch, state_all, out, stream);
}
