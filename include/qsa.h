/*
 * qsa.h -- C ABI of the B200 sparse-attention (QSA) library, libqsa.so.
 *
 * The library implements the four parts of QwFNfer's "Qwen Sparse Attention" node:
 *   1. the lightning indexer: each query scored against one mean-pooled, RMS-normed,
 *      IMRoPE'd key per block of `ratio` cells;
 *   2. top-k block selection plus a forced local window;
 *   3. block-sparse flash attention over the selected q8_0 or f16 KV rows;
 *   4. the pooled-key update when KV rows are appended.
 *
 * Reference interfaces replaced (paths inside the QwFNfer source tree):
 *   - graph_builder::sparse_attn_decode   src/qwfn_graph.cpp:450-546  -> qsa_decode
 *   - graph_builder::sparse_attn/qsa_top_k src/qwfn_graph.cpp:235-408 -> qsa_prefill
 *   - graph_builder::qsa_pool_rebuild      src/qwfn_graph.cpp:431-448 -> qsa_pool_rebuild
 *   - the K/V/raw-key writes (ggml_set_rows / ggml_cpy into the caches)
 *                                          src/qwfn_graph.cpp:466-469,504-528,249-254,349-360
 *                                                                     -> qsa_append
 *   - engine::qsa_decode_prepare / build_attn_inputs bias + table rules
 *                                          src/qwfn_engine.cpp:731-799,884-957
 *                                          (computed on the device from n_past; no host tables)
 *
 * Cache layouts are byte-identical to the reference:
 *   K, V   : per layer, n_ctx token rows of n_head_kv*head_dim elements in type_k/type_v,
 *            row t = head0[head_dim] head1[head_dim] ...   (src/qwfn_state.cpp:40-56)
 *            q8_0 = blocks of 32: { f16 d; int8 qs[32] }, 34 bytes, packed.
 *   idx    : F16 [n_ctx][idx_dim] raw (pre-norm, pre-rope) indexer keys   (src/qwfn_state.cpp:49)
 *   pool   : F16 [n_ctx/ratio][idx_dim] pooled+normed+roped block keys   (src/qwfn_engine.cpp:394-397)
 *
 * Conventions:
 *   - Every pointer that a kernel touches is a DEVICE pointer unless the comment says "host".
 *   - The caller owns every cache, input, output and workspace buffer.  No entry point allocates
 *     device memory, and none synchronises the stream except qsa_check and the *_sync helpers.
 *   - Work is stream-ordered on `stream`; calls on different streams over the same caches race.
 *   - Errors: an enum return.  Argument errors are found on the host (QSA_ERR_INVALID) before
 *     anything is launched.  Out-of-range values found on the device (for instance an n_past
 *     beyond n_ctx in a device-side table) are recorded in the workspace status word and the
 *     offending item is skipped; qsa_check() reads and clears it.  Nothing aborts.
 *   - Workspaces must be zeroed once (qsa_workspace_init) before first use; kernels leave the
 *     counters they use at zero again when they finish.
 */
#ifndef QSA_H
#define QSA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* cudaStream_t without requiring the CUDA headers. */
struct CUstream_st;
typedef struct CUstream_st * qsa_stream_t;

typedef enum qsa_status {
    QSA_OK              = 0,
    QSA_ERR_INVALID     = 1,  /* bad argument or descriptor (host-side check)            */
    QSA_ERR_CUDA        = 2,  /* a CUDA launch or copy failed                            */
    QSA_ERR_TIMEOUT     = 3,  /* a bounded device-side wait ran out                      */
    QSA_ERR_UNSUPPORTED = 4,  /* shape/type combination without a kernel                 */
    QSA_ERR_WORKSPACE   = 5,  /* workspace missing or smaller than *_workspace_size()    */
    QSA_ERR_DEVICE_ARG  = 6   /* an out-of-range value was found on the device           */
} qsa_status;

/* Element types, numbered as ggml numbers them (ggml_type). */
enum {
    QSA_TYPE_F32  = 0,
    QSA_TYPE_F16  = 1,
    QSA_TYPE_Q8_0 = 8,
    QSA_TYPE_BF16 = 30
};

/* Layer descriptor: the hyper-parameters of one QSA layer (src/qwfn_hparams.h:21-54). */
typedef struct qsa_desc {
    int32_t n_head;          /* query heads                                     (n_head)          */
    int32_t n_head_kv;       /* KV heads                                        (n_head_kv)       */
    int32_t head_dim;        /* 256                                             (n_embd_head_k)   */
    int32_t idx_n_head;      /* indexer heads                                   (idx_n_head)      */
    int32_t idx_dim;         /* indexer key length                              (idx_key_len)     */
    int32_t ratio;           /* cells per block r                               (compress_ratios) */
    int32_t top_k_blocks;    /* blocks kept by score                                              */
    int32_t window;          /* causal local window in tokens, forced at block granularity:
                                ceil(window/ratio)+1 blocks ending at the query's block.
                                0 = the reference rule: only the query's block, and only while it
                                is incomplete (src/qwfn_engine.cpp:936-950).                      */
    int32_t n_ctx;           /* cache capacity in tokens (a multiple of ratio)                    */
    int32_t type_k;          /* QSA_TYPE_Q8_0 or QSA_TYPE_F16                                     */
    int32_t type_v;          /* QSA_TYPE_Q8_0 or QSA_TYPE_F16                                     */
    int32_t rope_dim;        /* rotated dims of the indexer key (rope_dim)                        */
    int32_t sections[4];     /* IMRoPE sections (mrope_sections)                                  */
    float   rms_eps;         /* rms_eps                                                           */
    float   rope_freq_base;  /* rope_freq_base                                                    */
    const float * k_norm_w;  /* device [idx_dim], indexer.k_norm.weight; NULL means all ones      */
    uint32_t placement;      /* where the caches live (state_config's kv_host / idx_host,
                                src/qwfn_state.h:31-36): 0 = device memory, or QSA_KV_HOST and/or
                                QSA_IDX_HOST: pinned host memory mapped into the device's address
                                space (device-accessible at its host address), read and written by
                                the device over the bus.  The pooled keys stay in device memory.    */
} qsa_desc;

/* qsa_desc.placement bits. */
enum {
    QSA_KV_HOST  = 1u << 0,  /* K and V caches in pinned host memory */
    QSA_IDX_HOST = 1u << 1   /* raw indexer-key cache in pinned host memory */
};

/* One layer's caches of one sequence (device pointers, reference layouts above). */
typedef struct qsa_layer_cache {
    void     * k;
    void     * v;
    uint16_t * idx;
    uint16_t * pool;
} qsa_layer_cache;

/* One decode query, as a device-resident table entry: the query is token n_past of the
 * sequence whose caches are `cache`; after this step the cache holds n_past+1 tokens.
 * Kept in device memory so that a captured CUDA graph replays with new positions. */
typedef struct qsa_decode_item {
    qsa_layer_cache cache;
    int32_t n_past;
    int32_t reserved[3];
} qsa_decode_item;

/* ------------------------------------------------------------------ descriptors / sizes */
const char * qsa_status_string(qsa_status s);
/* Host-side validation of a descriptor against what the kernels support. */
qsa_status qsa_desc_check(const qsa_desc * d);
/* Blocks attended per query: top_k_blocks plus the forced-window blocks (KB). */
int32_t qsa_k_blocks(const qsa_desc * d);
/* Bytes of one cache row: which = 0 K, 1 V, 2 idx, 3 pool (per block). */
size_t qsa_row_bytes(const qsa_desc * d, int32_t which);
/* Bytes of one whole layer cache of n_ctx tokens: which as above. */
size_t qsa_cache_bytes(const qsa_desc * d, int32_t which);

/* ------------------------------------------------------------------ append / pool */
/* Write n_tok tokens at rows [pos0, pos0+n_tok): K and V (f32 [n_tok][n_head_kv*head_dim],
 * quantised to type_k/type_v with ggml's reference q8_0 rounding), the raw indexer key
 * (f32 [n_tok][idx_dim] -> F16), and the pooled key of every block that is complete at
 * pos0+n_tok and has a member in the range.  kidx may be NULL (no indexer write, no pool update).
 * Replaces the set_rows/cpy writes of src/qwfn_graph.cpp:466-476,504-528 and 249-254,349-360. */
qsa_status qsa_append(const qsa_desc * d, const qsa_layer_cache * cache /* host struct */,
                      int32_t pos0, int32_t n_tok,
                      const float * k, const float * v, const float * kidx,
                      qsa_stream_t stream);

/* Recompute pooled keys of blocks [blk0, blk0+n_blk) from the raw indexer cache.
 * pooled_f32 (optional, device [n_blk][idx_dim]) receives the f32 values before the F16 store.
 * Replaces graph_builder::qsa_pool_rebuild (src/qwfn_graph.cpp:412-448). */
qsa_status qsa_pool_rebuild(const qsa_desc * d, const qsa_layer_cache * cache /* host struct */,
                            int32_t blk0, int32_t n_blk, float * pooled_f32, qsa_stream_t stream);

/* ------------------------------------------------------------------ decode */
size_t qsa_decode_workspace_size(const qsa_desc * d, int32_t batch, int32_t max_n_kv);
/* Zero a workspace (required once before its first use). */
qsa_status qsa_workspace_init(void * ws, size_t ws_bytes, qsa_stream_t stream);

/* One decode step for `batch` queries (items: device table of qsa_decode_item).
 *   q      : [batch][n_head][head_dim], q_type QSA_TYPE_BF16 or QSA_TYPE_F32 (post-norm, post-rope)
 *   q_idx  : f32 [batch][idx_n_head][idx_dim]   indexer query (post q_norm and rope)
 *   k_new, v_new, kidx_new : f32 rows of the token being decoded, [batch][...] as in qsa_append;
 *            all three NULL = the caller already wrote row n_past (and the pooled keys)
 *   out    : f32 [batch][n_head][head_dim]
 *   sel_out: optional int32 [batch][KB]: selected block ids ascending, -1 padded
 * max_n_kv bounds n_past+1 over the batch (sizes the grid; a device value above it is an error).
 * Replaces graph_builder::sparse_attn_decode up to the output gate (src/qwfn_graph.cpp:450-541). */
qsa_status qsa_decode(const qsa_desc * d, const qsa_decode_item * items, int32_t batch, int32_t max_n_kv,
                      const void * q, int32_t q_type, const float * q_idx,
                      const float * k_new, const float * v_new, const float * kidx_new,
                      float * out, int32_t * sel_out,
                      void * ws, size_t ws_bytes, qsa_stream_t stream);

/* qsa_decode with the node's output gate applied where the attention stores its result: besides
 * (or, with out NULL, instead of) the f32 output, the call writes the gated product
 *   z = out * sigmoid(gate)        (ggml_mul(attn, ggml_sigmoid(gate)), f32, sigmoid 1/(1+exp(-g)))
 * gate: f32 [batch][n_head*head_dim] (qsa_front's gate), z: [batch][n_head*head_dim] as bf16
 * (z_type QSA_TYPE_BF16: rounded as the bf16 attn_output mul_mat converts it) or f32
 * (QSA_TYPE_F32, for q8_0 attn_output weights, which quantise it).  qsa_output_z then projects z.
 * Replaces graph_builder::sparse_attn_decode through the gate multiply (src/qwfn_graph.cpp:450-544). */
qsa_status qsa_decode_gated(const qsa_desc * d, const qsa_decode_item * items, int32_t batch, int32_t max_n_kv,
                            const void * q, int32_t q_type, const float * q_idx,
                            const float * k_new, const float * v_new, const float * kidx_new,
                            const float * gate, void * z, int32_t z_type, float * out /* optional */,
                            int32_t * sel_out, void * ws, size_t ws_bytes, qsa_stream_t stream);

/* The three stages of qsa_decode as separate calls (same arguments and workspace), for callers
 * that append elsewhere or time the stages: append (row n_past of each item, plus the pooled key
 * of a block it completes), select (scores + top-k into the workspace, optional sel_out),
 * attend (attention over the selection the last select left in the workspace). */
qsa_status qsa_decode_append(const qsa_desc * d, const qsa_decode_item * items, int32_t batch, int32_t max_n_kv,
                             const float * k_new, const float * v_new, const float * kidx_new,
                             void * ws, size_t ws_bytes, qsa_stream_t stream);
qsa_status qsa_decode_select(const qsa_desc * d, const qsa_decode_item * items, int32_t batch, int32_t max_n_kv,
                             const float * q_idx, int32_t * sel_out, void * ws, size_t ws_bytes, qsa_stream_t stream);
qsa_status qsa_decode_attend(const qsa_desc * d, const qsa_decode_item * items, int32_t batch, int32_t max_n_kv,
                             const void * q, int32_t q_type, float * out, void * ws, size_t ws_bytes,
                             qsa_stream_t stream);

/* qsa_decode without a caller workspace.  No counterpart in the reference.
 * For callers that cannot allocate device memory -- an operator run inside another framework's
 * planned graph sees only its input and output tensors, and a serving loop under a fixed memory
 * budget must not call cudaMalloc on the token path -- the scratch lives in a fixed device array
 * of 8 MiB inside the library (held on every GPU that loads it, until exit).  Arguments and
 * results are those of qsa_decode; a call whose qsa_decode_workspace_size() exceeds 8 MiB returns
 * QSA_ERR_WORKSPACE.  The first call on a device looks up the array's device address (a host-side
 * query, cudaGetSymbolAddress): make that first call before any stream capture.  Every call zeroes
 * the array's status word and counters on `stream` and otherwise reuses the last call's contents,
 * so calls that overlap on the GPU (other streams or threads) race; device-side range errors cannot
 * be read back through this entry point (the affected query's output is zero).  Nothing is
 * allocated. */
qsa_status qsa_decode_noalloc(const qsa_desc * d, const qsa_decode_item * items, int32_t batch, int32_t max_n_kv,
                              const void * q, int32_t q_type, const float * q_idx,
                              const float * k_new, const float * v_new, const float * kidx_new,
                              float * out, int32_t * sel_out, qsa_stream_t stream);

/* ------------------------------------------------------------------ KV-sequence-sharded decode
 * No counterpart in the reference, which decodes a sequence on one device: for contexts whose
 * caches do not fit (or are not fast enough on) one GPU, the cells of every layer are split into
 * contiguous block ranges, one per GPU.  Shard g holds blocks [blk_lo, blk_hi) (cells
 * blk_lo*ratio .. blk_hi*ratio-1) in local arrays: the caches named by `items` on that GPU have
 * row 0 = cell blk_lo*ratio and pooled row 0 = block blk_lo.  The descriptor (n_ctx included),
 * n_past and max_n_kv stay global.  One step, on every shard with the same arguments otherwise:
 *   1. qsa_shard_candidates: append of the new token by the shard holding its cell (the others
 *      skip it), scores of the shard's visible blocks, and the shard's best KB blocks outside the
 *      forced window, into cand = int32 [2][batch][KB]: the block ids (-1 padded), then the bits
 *      of their f32 scores.
 *   2. the caller all-gathers cand, in shard order: all_cand = int32 [n_shards][2][batch][KB].
 *   3. qsa_shard_attend: the global selection (identical to qsa_decode's; sel_out optional,
 *      [batch][KB] ascending), then attention over the shard's part of it into `state`,
 *      f32 [batch][qsa_shard_state_floats()]: per (KV head x 8) row its running max (log2
 *      domain), its sum of weights, and its unnormalised output.
 *   4. the caller all-gathers the states: [n_shards][batch][...].
 *   5. qsa_merge_states: out f32 [batch][n_head][head_dim], as qsa_decode's.
 * Workspaces are sized by qsa_shard_workspace_size with the global max_n_kv and the shard's
 * block range (the attention's split over CTAs follows the shard's expected share of blocks). */
size_t qsa_shard_state_floats(const qsa_desc * d);
/* The same decode with the indexer caches replicated: every rank holds the raw keys and pooled keys
 * of all blocks (global rows) and only the K/V rows of blocks [blk_lo, blk_hi) (row 0 = cell
 * blk_lo * ratio).  Every rank then computes the identical global selection itself, so a step is
 * qsa_shard_decode_ri (append, selection, attention over the shard's selected blocks into
 * `state`), one all-gather of the states and qsa_merge_states: one exchange instead of two.
 * Workspaces: qsa_shard_workspace_size.  qsa_shard_append_ri writes rows [pos0, pos0+n_tok): every
 * raw key (and the pooled keys of the blocks they complete), the K/V rows inside the shard. */
qsa_status qsa_shard_append_ri(const qsa_desc * d, const qsa_layer_cache * cache /* host struct */,
                               int32_t blk_lo, int32_t blk_hi, int32_t pos0, int32_t n_tok,
                               const float * k, const float * v, const float * kidx, qsa_stream_t stream);
qsa_status qsa_shard_decode_ri(const qsa_desc * d, const qsa_decode_item * items, int32_t batch, int32_t max_n_kv,
                               int32_t blk_lo, int32_t blk_hi, const void * q, int32_t q_type, const float * q_idx,
                               const float * k_new, const float * v_new, const float * kidx_new, float * state,
                               int32_t * sel_out, void * ws, size_t ws_bytes, qsa_stream_t stream);
size_t qsa_shard_workspace_size(const qsa_desc * d, int32_t batch, int32_t max_n_kv, int32_t blk_lo, int32_t blk_hi);
/* qsa_append into a shard's local arrays: global rows [pos0, pos0+n_tok), all inside the shard's
 * cells; pooled keys carry their global block positions. */
qsa_status qsa_shard_append(const qsa_desc * d, const qsa_layer_cache * cache /* host struct */,
                            int32_t blk_lo, int32_t blk_hi, int32_t pos0, int32_t n_tok,
                            const float * k, const float * v, const float * kidx, qsa_stream_t stream);
qsa_status qsa_shard_candidates(const qsa_desc * d, const qsa_decode_item * items, int32_t batch, int32_t max_n_kv,
                                int32_t blk_lo, int32_t blk_hi, const float * q_idx,
                                const float * k_new, const float * v_new, const float * kidx_new,
                                int32_t * cand, void * ws, size_t ws_bytes, qsa_stream_t stream);
qsa_status qsa_shard_attend(const qsa_desc * d, const qsa_decode_item * items, int32_t batch, int32_t max_n_kv,
                            int32_t blk_lo, int32_t blk_hi, int32_t n_shards, const int32_t * all_cand,
                            int32_t cand_stride /* int32 between shards' slices; 0 = 2*batch*KB */,
                            const void * q, int32_t q_type, float * state,
                            int32_t * sel_out, void * ws, size_t ws_bytes, qsa_stream_t stream);
qsa_status qsa_merge_states(const qsa_desc * d, int32_t n_parts, int32_t batch, const float * states, float * out,
                            qsa_stream_t stream);

/* The whole sharded step on one rank, the two exchanges done with the caller's NCCL communicator
 * (the ncclComm_t of the ranks holding the shards; shard order = rank order in it, n_ranks its size):
 *   index_replicated 0: qsa_shard_candidates -> ncclAllGather -> qsa_shard_attend
 *   index_replicated 1: qsa_shard_decode_ri (indexer caches replicated on every rank)
 * then ncclAllGather of the states and qsa_merge_states into out (f32 [batch][n_head][head_dim],
 * identical on every rank; sel_out optional).  All work is stream-ordered on `stream`.  NCCL is
 * not linked by the library: the entry points come from the libnccl.so.2 already loaded in the
 * process (QSA_ERR_UNSUPPORTED if none is).  The workspace (qsa_decode_sharded_workspace_size,
 * zeroed once) holds the shard calls' workspace and the gathered candidates and states.
 * Replaces graph_builder::sparse_attn_decode (src/qwfn_graph.cpp:450-541) for a sequence whose
 * cells are split over ranks; the exchange itself has no counterpart in the reference. */
typedef struct ncclComm * qsa_nccl_comm_t;      /* ncclComm_t */
size_t qsa_decode_sharded_workspace_size(const qsa_desc * d, int32_t batch, int32_t max_n_kv,
                                         int32_t blk_lo, int32_t blk_hi, int32_t n_ranks);
qsa_status qsa_decode_sharded(const qsa_desc * d, const qsa_decode_item * items, int32_t batch, int32_t max_n_kv,
                              int32_t blk_lo, int32_t blk_hi, int32_t index_replicated,
                              qsa_nccl_comm_t comm, int32_t n_ranks,
                              const void * q, int32_t q_type, const float * q_idx,
                              const float * k_new, const float * v_new, const float * kidx_new,
                              float * out, int32_t * sel_out, void * ws, size_t ws_bytes, qsa_stream_t stream);

/* ------------------------------------------------------------------ all-gather over peer memory
 * The two exchanges of the sharded decode without a collective library: every rank owns a gather
 * buffer of qsa_peer_buffer_bytes(n_ranks, slot_bytes) bytes ([n_ranks][slot_bytes] + flags,
 * zeroed once) and maps the buffers of all ranks through CUDA IPC.  qsa_peer_push stores this
 * rank's slice (`slot_bytes`, a multiple of 16, from `src`) into slot `rank` of every buffer (`bufs`:
 * a device array of the n_ranks buffer addresses, this rank's own among them) over NVLink, then
 * publishes it with a release flag carrying the round's epoch (`epoch`, `counter`: two zeroed device
 * uint32 per buffer, owned by this rank).  qsa_peer_wait returns once all n_ranks slices of the
 * round are in this rank's buffer (bounded wait: QSA_ERR_TIMEOUT through the status word of `ws`,
 * read by qsa_check).  slot_bytes is a multiple of 4; slots start at a stride rounded up to 16
 * bytes; n_ranks is at most 32.  All ranks must push and wait on a buffer in the same order.
 * A push overwrites the peers' slots without waiting for them to finish reading the previous
 * round, so a caller alternates at least two buffers (channels): a rank pushes into a channel
 * again only after a wait on another channel, which the peers' own pushes (made after they
 * consumed this channel) complete.  No counterpart in the reference. */
qsa_status qsa_ipc_handle(const void * ptr, void * handle /* host, 64 bytes */, size_t * offset /* host */);
qsa_status qsa_ipc_open(const void * handle /* host, 64 bytes */, void ** base /* host */);
qsa_status qsa_ipc_close(void * base);
size_t qsa_peer_buffer_bytes(int32_t n_ranks, size_t slot_bytes);
qsa_status qsa_peer_push(void * const * bufs, int32_t n_ranks, int32_t rank, const void * src, size_t slot_bytes,
                         uint32_t * epoch, uint32_t * counter, qsa_stream_t stream);
qsa_status qsa_peer_wait(const void * local_buf, int32_t n_ranks, size_t slot_bytes, const uint32_t * epoch,
                         void * ws, size_t ws_bytes, qsa_stream_t stream);

/* The replicated-index step with its state exchange fused into the kernels (no push or wait
 * launch): one channel of the peer buffers above, as this rank sees it.  region[p] is rank p's
 * gather buffer of the channel (this rank's own, or its CUDA IPC mapping), laid out as
 * qsa_peer_buffer_bytes(n_ranks, slot_bytes) with slot_bytes = batch * qsa_shard_state_floats * 4;
 * epoch is this rank's zeroed device counter of the channel.  At most 8 ranks. */
typedef struct qsa_peer_slots {
    void * region[8];
    int32_t n_ranks;
    int32_t rank;
    uint32_t * epoch;
} qsa_peer_slots;

/* qsa_shard_decode_ri whose attention (or its merge) stores this rank's state into slot `rank` of
 * every region over NVLink, after which a one-warp kernel publishes it (the channel's next epoch,
 * a system-scope release flag in every region).  qsa_merge_states_peer then waits (bounded:
 * QSA_ERR_TIMEOUT through the status word of `ws`, at least 16 bytes, read by qsa_check) until
 * every rank's state of the round is in this rank's region and merges them in rank order into out
 * (f32 [batch][n_head][head_dim]).  Consecutive steps alternate two channels, as for
 * qsa_peer_push: a rank stores into a channel again only after every peer has read it. */
qsa_status qsa_shard_decode_ri_peer(const qsa_desc * d, const qsa_decode_item * items, int32_t batch, int32_t max_n_kv,
                                    int32_t blk_lo, int32_t blk_hi, const void * q, int32_t q_type, const float * q_idx,
                                    const float * k_new, const float * v_new, const float * kidx_new,
                                    const qsa_peer_slots * slots, int32_t * sel_out, void * ws, size_t ws_bytes,
                                    qsa_stream_t stream);
qsa_status qsa_merge_states_peer(const qsa_desc * d, const qsa_peer_slots * slots, int32_t batch, float * out,
                                 void * ws, size_t ws_bytes, qsa_stream_t stream);

/* ------------------------------------------------------------------ prefill */
size_t qsa_prefill_workspace_size(const qsa_desc * d, int32_t T, int32_t max_n_kv);

/* Chunked prefill of T tokens at positions [n_past, n_past+T) of one sequence: append K/V/raw
 * keys, update the pooled keys of the blocks completed, score every query against the blocks
 * complete at its position, select, and attend.  Inputs are laid out as in qsa_decode with
 * `batch` replaced by T.  k_new/v_new/kidx_new NULL = already appended.
 * Replaces graph_builder::sparse_attn + qsa_top_k (src/qwfn_graph.cpp:235-408) together with
 * the per-chunk host inputs of engine::build_attn_inputs (src/qwfn_engine.cpp:884-957): the
 * result does not depend on how the caller chunks the T tokens. */
qsa_status qsa_prefill(const qsa_desc * d, const qsa_layer_cache * cache /* host struct */,
                       int32_t n_past, int32_t T,
                       const void * q, int32_t q_type, const float * q_idx,
                       const float * k_new, const float * v_new, const float * kidx_new,
                       float * out, int32_t * sel_out,
                       void * ws, size_t ws_bytes, qsa_stream_t stream);

/* qsa_prefill with the output gate applied in the attention's final store, as qsa_decode_gated
 * (arguments as there, `batch` replaced by T).  Replaces graph_builder::sparse_attn through the gate
 * multiply (src/qwfn_graph.cpp:235-405). */
qsa_status qsa_prefill_gated(const qsa_desc * d, const qsa_layer_cache * cache /* host struct */,
                             int32_t n_past, int32_t T,
                             const void * q, int32_t q_type, const float * q_idx,
                             const float * k_new, const float * v_new, const float * kidx_new,
                             const float * gate, void * z, int32_t z_type, float * out /* optional */,
                             int32_t * sel_out, void * ws, size_t ws_bytes, qsa_stream_t stream);

/* ------------------------------------------------------------------ projection front */
/* The projections feeding the node, as graph_builder::sparse_attn_decode builds them
 * (src/qwfn_graph.cpp:465, 479-484, 505-518; prefill :324-347).  Weights are row-major
 * [out][n_embd] (ggml's mul_mat layout), 16-byte aligned, in one of two formats (w_type):
 *   QSA_TYPE_BF16  bf16 values; the activations are rounded to bf16 (ggml's vec_dot_bf16);
 *   QSA_TYPE_Q8_0  q8_0 rows of n_embd/32 blocks {f16 d; int8 qs[32]} (34 bytes); the activations
 *                  are quantised to q8_0 with ggml's reference rounding and each block contributes
 *                  its integer dot times f32(d_w) * f32(d_x) (ggml_vec_dot_q8_0_q8_0).
 * The norm weights are f32. */
typedef struct qsa_front_weights {
    const void  * wq;          /* attn_q.weight [2*head_dim*n_head][n_embd]: head h's query rows
                                  [2*h*hd, 2*h*hd + hd), its gate rows the next hd */
    const void  * wk;          /* attn_k.weight [head_dim*n_head_kv][n_embd] */
    const void  * wv;          /* attn_v.weight [head_dim*n_head_kv][n_embd] */
    const void  * wq_idx;      /* indexer.q_proj.weight [idx_dim*idx_n_head][n_embd] */
    const void  * wk_idx;      /* indexer.k_proj.weight [idx_dim][n_embd] */
    const float * q_norm;      /* attn_q_norm.weight [head_dim] (NULL = 1) */
    const float * k_norm;      /* attn_k_norm.weight [head_dim] (NULL = 1) */
    const float * q_idx_norm;  /* indexer.q_norm.weight [idx_dim] (NULL = 1) */
    int32_t       n_embd;      /* model width: at most 12288; a multiple of 8 (bf16) or of 256 (q8_0) */
    int32_t       w_type;      /* QSA_TYPE_BF16 or QSA_TYPE_Q8_0 (all five matrices) */
} qsa_front_weights;

size_t qsa_front_workspace_size(const qsa_desc * d, const qsa_front_weights * w, int32_t T);
/* For T tokens at positions pos[T] (device int32) with activations x [T][n_embd] (device f32):
 *   y = W x in f32 (the weight format's products above);
 *   q_out     f32 [T][n_head][head_dim]      rms_norm * q_norm, IMRoPE at pos
 *   gate_out  f32 [T][n_head*head_dim]       the gate half of attn_q, raw
 *   q_idx_out f32 [T][idx_n_head][idx_dim]   rms_norm * q_idx_norm, IMRoPE at pos
 *   k_out     f32 [T][n_head_kv*head_dim]    rms_norm * k_norm, IMRoPE at pos
 *   v_out     f32 [T][n_head_kv*head_dim]    raw
 *   kidx_out  f32 [T][idx_dim]               raw (normed and roped when pooled)
 * which are qsa_decode's q (QSA_TYPE_F32), q_idx, k_new, v_new and kidx_new.  Up to 16 tokens the
 * projections stream the weights (a matrix-vector kernel per group of 4 tokens); above, with
 * rope_dim a multiple of 64, they run as one tcgen05 GEMM whose epilogue applies the norms and
 * IMRoPE (f32 accumulation in the tensor cores; q8_0 weights and activations enter it as f16 of
 * their d * q values, each rounded once).  The workspace is zeroed once (qsa_workspace_init) and
 * 16-byte aligned (QSA_ERR_WORKSPACE).  Replaces the projection, norm and rope nodes of
 * src/qwfn_graph.cpp:465, 479-484, 505-518. */
qsa_status qsa_front(const qsa_desc * d, const qsa_front_weights * w, int32_t T, const int32_t * pos,
                     const float * x, float * q_out, float * gate_out, float * q_idx_out,
                     float * k_out, float * v_out, float * kidx_out,
                     void * ws, size_t ws_bytes, qsa_stream_t stream);

/* The output side of the node (src/qwfn_graph.cpp:543-545; prefill :406-407): for T tokens
 *   y = attn_output.weight * (attn * sigmoid(gate)),
 * sigmoid 1/(1+exp(-g)) in f32; the gated product enters the weight format's products as qsa_front's
 * activations do.  wo: [n_embd][n_head*head_dim] in bf16 or q8_0 (w_type, 16-byte aligned); attn:
 * f32 [T][n_head][head_dim] (qsa_decode's out); gate: f32 [T][n_head*head_dim] (qsa_front's gate);
 * y: f32 [T][n_embd].  Up to 16 tokens no workspace is used (ws may be NULL); above, the tokens run
 * as one tcgen05 GEMM and ws holds qsa_output_workspace_size(d, n_embd, w_type, T) bytes (16-byte
 * aligned, zeroed once, else QSA_ERR_WORKSPACE); n_embd is then a multiple of 4 and y 16-byte
 * aligned. */
size_t qsa_output_workspace_size(const qsa_desc * d, int32_t n_embd, int32_t w_type, int32_t T);
qsa_status qsa_output(const qsa_desc * d, const void * wo, int32_t n_embd, int32_t w_type, int32_t T,
                      const float * attn, const float * gate, float * y, void * ws, size_t ws_bytes,
                      qsa_stream_t stream);
/* The attn_output projection of a gated product written by qsa_decode_gated / qsa_prefill_gated:
 * y = attn_output.weight * z, z [T][n_head*head_dim] bf16 (z_type QSA_TYPE_BF16, bf16 weights only:
 * the GEMM path reads it as its operand, no gate pass) or f32 (QSA_TYPE_F32, either weight type).
 * Workspace, alignment and paths as qsa_output (src/qwfn_graph.cpp:545; prefill :406-407). */
qsa_status qsa_output_z(const qsa_desc * d, const void * wo, int32_t n_embd, int32_t w_type, int32_t T,
                        const void * z, int32_t z_type, float * y, void * ws, size_t ws_bytes, qsa_stream_t stream);

/* ------------------------------------------------------------------ descriptors from GGUF metadata */
/* The node's hyper-parameters of a GGUF file, read as model_index::read_metadata reads them
 * (src/qwfn_model.cpp:111-152): keys under "<arch>." with the same defaults; integer keys of any
 * integer type, f32 keys only as F32, arrays of 32/64-bit integers.  Only "qwen4exp" files are
 * accepted (QSA_ERR_UNSUPPORTED otherwise), as the reference loader does. */
#define QSA_GGUF_MAX_LAYERS 256
typedef struct qsa_gguf_hparams {
    char    arch[64];
    int32_t n_layer, n_embd, n_ctx_train;
    int32_t n_head, n_head_kv, head_dim;
    float   rms_eps;
    int32_t full_attention_interval;
    int32_t n_compress;                               /* entries of attention.compress_ratios */
    int32_t compress_ratios[QSA_GGUF_MAX_LAYERS];     /* per layer; 0 = a dense attention layer */
    float   rope_freq_base;
    int32_t rope_dim;
    int32_t sections[4];
    int32_t idx_n_head, idx_dim, idx_top_k;
} qsa_gguf_hparams;

/* Read the metadata of the GGUF file at `path` (host path; tensor data is not read).  err (host,
 * err_len bytes, optional) receives a message on failure. */
qsa_status qsa_gguf_read_hparams(const char * path, qsa_gguf_hparams * hp, char * err, size_t err_len);
/* 1 when layer il runs the node: an attention layer ((il + 1) % full_attention_interval == 0,
 * hparams::is_attn_layer) with compress_ratios[il] > 0; 0 otherwise. */
int32_t qsa_gguf_is_qsa_layer(const qsa_gguf_hparams * hp, int32_t il);
/* The descriptor of sparse-attention layer il for a cache of n_ctx cells (rounded up to whole
 * blocks): ratio compress_ratios[il], top_k_blocks = ceil((idx_top_k + r - 1) / r) - 1 with the
 * window rule given (0 = the reference's: its incomplete block forced, engine::init,
 * src/qwfn_engine.cpp:384-431).  Returns qsa_desc_check's verdict on it (the descriptor is filled
 * in either way); QSA_ERR_INVALID when il is not such a layer. */
qsa_status qsa_gguf_layer_desc(const qsa_gguf_hparams * hp, int32_t il, int32_t n_ctx, int32_t window,
                               int32_t type_k, int32_t type_v, const float * k_norm_w, qsa_desc * out);

/* ------------------------------------------------------------------ staging */
/* Copy `bytes` (a multiple of 16, both addresses 16-byte aligned) from src to dst with a kernel on
 * `stream`, chained to the kernels around it by programmatic dependent launch.  Each side is device
 * memory of the current device, managed memory, or pinned host memory mapped at its host address
 * (QSA_ERR_INVALID otherwise).  Moves a decode step's activations in and its output out without a
 * copy-engine hand-over; replaces the per-token ggml_backend_tensor_set of the decode inputs
 * (src/qwfn_engine.cpp:738-753) and the read of the result after the graph computes. */
qsa_status qsa_stage_copy(void * dst, const void * src, size_t bytes, qsa_stream_t stream);

/* ------------------------------------------------------------------ status */
/* Synchronise `stream`, read and clear the workspace status word. */
qsa_status qsa_check(void * ws, size_t ws_bytes, qsa_stream_t stream);

/* Library version (major*10000 + minor*100 + patch) and the device kernels' target. */
int32_t qsa_version(void);

#ifdef __cplusplus
}
#endif
#endif /* QSA_H */
