// qsa_kernels.cuh -- kernel entry points of libqsa and their launch constants.
#pragma once
#include <atomic>

#include "qsa_common.cuh"

namespace qsa {

// Runs `set` (cudaFuncSetAttribute calls) once on each device: function attributes are a
// per-device setting, so a process driving several GPUs sets them on every device it launches
// on.  `done` holds one bit per device id; the calls are idempotent, so two threads racing on a
// device's first launch both just set them.
template <typename F>
cudaError_t once_per_device(std::atomic<uint64_t> & done, F && set) {
    int dev = -1;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    const uint64_t bit = 1ull << dev;
    if (done.load(std::memory_order_acquire) & bit) return cudaSuccess;
    e = set();
    if (e == cudaSuccess) done.fetch_or(bit, std::memory_order_acq_rel);
    return e;
}

constexpr int MAX_KB = 1024;          // blocks kept per query that the kernels can hold
constexpr int SEL_THREADS_HOST = 512;       // threads of a scoring/selection CTA

__global__ void append_rows_kernel(DevDesc d, qsa_layer_cache c, int pos0,
        const float * k, const float * v, const float * kidx);
__global__ void pool_blocks_kernel(DevDesc d, const uint16_t * idx, uint16_t * pool, int blk0, int n_blk, float * out_f32);
__global__ void append_decode_kernel(DevDesc d, const qsa_decode_item * items,
        const float * k, const float * v, const float * kidx, uint32_t * status);
constexpr int APPEND_DECODE_THREADS = 1024;
// dynamic shared memory of append_decode_kernel: one block of raw indexer keys
inline size_t append_decode_smem(const DevDesc & d) { return (size_t) d.ratio * MAX_IDX_DIM * 2; }

__global__ void score_select_kernel(DevDesc d, const qsa_decode_item * items, const uint16_t * pool0, int n_past0,
        const float * q_idx, int blocks_per_cta, float * scores_ws, int scores_stride, unsigned * counters,
        int * sel_ws, int * nsel_ws, int * sel_out, uint32_t * status, float * cand_scores);

// Leading bytes of a decode workspace that must be zero before a call (status word + counters).
size_t decode_workspace_zero_prefix(const qsa_desc * d, int32_t batch, int32_t max_n_kv);
// The kernels' view of a descriptor that passed qsa_desc_check (derived values filled in).
DevDesc dev_desc(const qsa_desc * d);

// Host launcher of the attention kernel and, when a query spans several CTAs (max_chunks > 1),
// of the merge of their partials (defined beside the kernels).  chained: a kernel of the same call
// precedes the attention, which may then start early (programmatic launch); otherwise it is an
// ordinary launch that waits for all earlier work in the stream.
cudaError_t launch_attn(const DevDesc & d, cudaStream_t st, bool chained, int n_q, const qsa_decode_item * items,
        qsa_layer_cache cache0, int n_past0, const void * q, int q_type, const int * sel_ws, const int * nsel_ws,
        int tiles_per_cta, int max_chunks, float * part_o, float * part_ml, OutSpec outs, uint32_t * status,
        const StateDst & sdst);
cudaError_t attn_set_attrs();
// Cells per attention tile.
int attn_tile_cells();
// Rows (KV head x query head) of the attention state: a partial is rows x head_dim floats.
int attn_state_rows();
// Attention CTAs resident on the GPU at once for a KV type (the CTAs of one wave).
int attn_resident_ctas(int type_k);

// Prefill indexer scores on tcgen05 (idx_n_head 1, 2 or 4) and the warp-per-query selection over
// precomputed scores (qsa_prefill_tc.cu).
cudaError_t launch_prefill_scores_tc(const DevDesc & d, cudaStream_t st, const float * q_idx, int T,
                                     const uint16_t * pool, int n_blocks, float * scores, int scores_stride,
                                     uint32_t * status);
cudaError_t launch_select_scores_warp(const DevDesc & d, cudaStream_t st, int n_past0, int T, const float * scores,
                                      int scores_stride, int * sel_ws, int * nsel_ws, int * sel_out, uint32_t * status);

// KV-stationary prefill attention on tcgen05 (qsa_prefill_attn.cu): q8_0, ratio 64, 8 query heads
// per KV head.  Workspace: prefill_kv_workspace bytes at `ws`.
bool prefill_kv_supported(const DevDesc & d, int T);
size_t prefill_kv_workspace(const DevDesc & d, int T, int n_blocks);
cudaError_t launch_prefill_attn_kv(const DevDesc & d, cudaStream_t st, qsa_layer_cache cache, int n_past0, int T,
                                   const void * q, int q_type, const int * sel, const int * nsel, int n_blocks,
                                   unsigned char * ws, OutSpec outs, uint32_t * status);

// The prefill-sized projections on tcgen05 (qsa_proj_gemm.cu).  Front: xb [T][n_embd] 16-bit
// activations, w[5] the 16-bit weights (attn_q, attn_k, attn_v, indexer.q_proj, indexer.k_proj),
// cs [T][rope_dim/2] the tokens' rope table, norm[3] (q, k, q_idx; null = 1), out[6] = q, gate,
// q_idx, k, v, kidx.  Plain: y[T][N] = a16[T][K] w[N][K]^T.  f16 selects f16 operands (else bf16).
int proj_front_tiles(const DevDesc & d);
cudaError_t launch_proj_gemm_front(const DevDesc & d, cudaStream_t st, int T, int n_embd, const void * xb,
                                   const void * const w[5], bool f16, const float2 * cs, const float * const norm[3],
                                   float * const out[6], uint32_t * status);
cudaError_t launch_proj_gemm_plain(cudaStream_t st, int T, int K, int N, const void * a16, const void * w, bool f16,
                                   float * y, uint32_t * status);

// KV-sequence-sharded decode: global selection from all shards' candidates, and the log-sum-exp
// merge of the shards' attention states (qsa_shard.cu).
cudaError_t launch_shard_select(const DevDesc & d, cudaStream_t st, const qsa_decode_item * items, int n_shards,
        int batch, const int * cand, size_t cand_stride, int blo, int bhi, int * sel_out, int * sel_ws, int * nsel_ws,
        uint32_t * status);
// flags != null: first wait (bounded; DEV_TIMEOUT in status) until flags[0..n_parts) reach *epoch
// (the peer exchange's publication), then read the states through L2.
cudaError_t launch_merge_states(const DevDesc & d, cudaStream_t st, int n_parts, int batch, const float * states,
        float * out, const uint32_t * flags = nullptr, const uint32_t * epoch = nullptr, uint32_t * status = nullptr);
// Publication of states stored into every rank's gather region (qsa_peer.cu): launched
// programmatically behind the kernel that stored them, it advances *epoch and sets this rank's
// flag in every region (flag[p], p < n) to it with a system-scope release.
cudaError_t launch_peer_publish(cudaStream_t st, uint32_t * const * flag, int n, uint32_t * epoch);

}  // namespace qsa
