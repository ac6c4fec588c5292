// qsa_api.cu -- the C ABI of libqsa (include/qsa.h): validation, workspace layout, launches.
#include <climits>
#include <cmath>
#include <cstdlib>
#include <cstring>

#include "qsa_kernels.cuh"

namespace qsa {
namespace {


inline int ceil_div(int64_t a, int64_t b) { return (int) ((a + b - 1) / b); }

int n_force_of(const qsa_desc * d) { return d->window > 0 ? ceil_div(d->window, d->ratio) + 1 : 1; }

size_t kv_row_bytes(int type, int64_t n) {
    return type == QSA_TYPE_Q8_0 ? (size_t) (n / QK8_0) * Q8_0_BYTES : (size_t) n * 2;
}

DevDesc make_dev(const qsa_desc * d) {
    DevDesc x;
    std::memset(&x, 0, sizeof x);
    x.n_head = d->n_head; x.n_head_kv = d->n_head_kv; x.head_dim = d->head_dim;
    x.gqa = d->n_head / d->n_head_kv;
    x.idx_n_head = d->idx_n_head; x.idx_dim = d->idx_dim; x.ratio = d->ratio;
    x.top_k = d->top_k_blocks; x.n_force = n_force_of(d); x.kb = x.top_k + x.n_force; x.window = d->window;
    x.n_ctx = d->n_ctx; x.type_k = d->type_k; x.type_v = d->type_v; x.rope_dim = d->rope_dim;
    for (int i = 0; i < 4; i++) x.sections[i] = d->sections[i];
    x.rms_eps = d->rms_eps;
    x.theta_scale = powf(d->rope_freq_base, -2.0f / (float) d->rope_dim);   // as ggml's rope computes it
    x.inv_ratio = 1.0f / (float) d->ratio;
    x.scale_log2 = (float) (1.4426950408889634 / std::sqrt((double) d->head_dim));
    x.k_norm_w = d->k_norm_w;
    const int64_t kv_dim = (int64_t) d->n_head_kv * d->head_dim;
    x.rb_k = (int64_t) kv_row_bytes(d->type_k, kv_dim);
    x.rb_v = (int64_t) kv_row_bytes(d->type_v, kv_dim);
    x.hb_k = (int) kv_row_bytes(d->type_k, d->head_dim);
    x.hb_v = (int) kv_row_bytes(d->type_v, d->head_dim);
    x.shard_blk0 = 0;
    x.shard_blk1 = INT_MAX;
    x.kv_host = (d->placement & QSA_KV_HOST) ? 1 : 0;
    return x;
}

struct WsLayout {
    size_t status, cnt_sel, scores, sel, nsel, part_o, part_ml, total;
    int scores_stride, max_chunks, tiles_per_cta;
};

size_t align256(size_t x) { return (x + 255) & ~(size_t) 255; }

constexpr int ATTN_TWO_TILE_MIN = 64;          // tiles of a query from which a CTA takes two

WsLayout ws_layout(const DevDesc & d, int n_q, int max_n_kv) {
    WsLayout w;
    w.scores_stride = std::max(4, ceil_div(ceil_div(max_n_kv, d.ratio), 4) * 4);   // 16-byte rows
    const int max_tiles = std::max(1, ceil_div((int64_t) d.kb * d.ratio, attn_tile_cells()));
    // Tiles a query is expected to have here: all of them, or on a KV shard its share of the
    // visible blocks (selections are spread over the sequence) plus the window, which its tail
    // shard holds.  The grid still covers max_tiles; chunks past a query's tiles exit at once.
    int exp_tiles = max_tiles;
    if (d.shard_blk0 > 0 || d.shard_blk1 != INT_MAX) {
        const int64_t n_blk = std::max(1, ceil_div(max_n_kv, d.ratio));
        const int64_t mine = std::max<int64_t>(0, std::min<int64_t>(d.shard_blk1, n_blk) - d.shard_blk0);
        exp_tiles = std::min<int64_t>(max_tiles, ceil_div((int64_t) max_tiles * mine, n_blk) +
                                                     ceil_div((int64_t) d.n_force * d.ratio, attn_tile_cells()));
        exp_tiles = std::max(1, exp_tiles);
    }
    // Chunks (CTAs) per query: while every tile of the batch fits one wave of attention CTAs
    // (latency), one tile each for short queries and two for long ones (the second tile's rows
    // arrive while the first is computed, and the merge reads half the partials: config 2's step
    // 0.9 us shorter); otherwise as many chunks as one wave gives each query.
    const int wave = attn_resident_ctas(d.type_k);
    int tpc;
    if ((int64_t) n_q * exp_tiles <= wave) {
        tpc = exp_tiles >= ATTN_TWO_TILE_MIN ? 2 : 1;
    } else {
        const int nch = std::min(std::max(1, wave / n_q), exp_tiles);
        tpc = ceil_div(exp_tiles, nch);
    }
    tpc = std::min(tpc, max_tiles);
    w.tiles_per_cta = tpc;
    w.max_chunks = ceil_div(max_tiles, tpc);
    size_t o = 0;
    w.status  = o; o = align256(o + 16);
    w.cnt_sel = o; o = align256(o + (size_t) n_q * 4);
    w.scores  = o; o = align256(o + (size_t) n_q * w.scores_stride * 4);
    w.sel     = o; o = align256(o + (size_t) n_q * d.kb * 4);
    w.nsel    = o; o = align256(o + (size_t) n_q * 4);
    const size_t parts = w.max_chunks > 1 ? (size_t) n_q * w.max_chunks : 0;   // one partial per CTA
    w.part_o  = o; o = align256(o + parts * attn_state_rows() * HEAD_DIM * 4);
    w.part_ml = o; o = align256(o + parts * 2 * attn_state_rows() * 4);
    w.total = o;
    return w;
}

qsa_status cuda_status(cudaError_t e) { return e == cudaSuccess ? QSA_OK : QSA_ERR_CUDA; }

std::atomic<uint64_t> attrs_done{0};
qsa_status set_attrs() {
    return cuda_status(once_per_device(attrs_done, [] {
        cudaError_t e = attn_set_attrs();
        if (e == cudaSuccess)
            e = cudaFuncSetAttribute(score_select_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 160 * 1024);
        if (e == cudaSuccess)
            e = cudaFuncSetAttribute(append_decode_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 64 * 1024);
        return e;
    }));
}

// Launch chaining.  Kernels after the first of a call are launched programmatically: they may
// start before the kernel ahead of them ends, and read what it writes only after pdl_wait, but
// read the call's inputs (items, q, q_idx, caches) at once.  That is safe because the first kernel
// of every call starts its dependents only once all earlier work in the stream is complete,
// whatever that work is (the caller's kernels, qsa_stage_copy, another call): it is an ordinary
// launch, or (the decode append) it waits for the kernel ahead before it reads anything or
// triggers.  `chained`: a kernel of the same call precedes this launch.

// Scores + selection into the workspace (and sel_out).  Sharded (cand_scores != null): scores of
// the shard's blocks only, and its candidates with their scores in sel_out / cand_scores.
qsa_status launch_select(const DevDesc & d, const WsLayout & w, int n_q, const qsa_decode_item * items,
                         qsa_layer_cache cache0, int n_past0, const float * q_idx, int32_t * sel_out,
                         unsigned char * ws, cudaStream_t st, bool chained, float * cand_scores = nullptr) {
    uint32_t * status = reinterpret_cast<uint32_t *>(ws + w.status);
    // blocks per scoring CTA: the fewest (whole row pairs of every warp, at least one) that keep
    // the batch's scoring grid within one wave (a CTA holds a whole SM's registers: one wave is
    // 148 CTAs); a second wave would start its CTAs only when the first leaves
    const int lo = d.shard_ri ? 0 : d.shard_blk0, hi = d.shard_ri ? INT_MAX : d.shard_blk1;
    const int n_blk = std::max(1, std::min(w.scores_stride, hi) - lo);   // blocks scored
    constexpr int PAIRS = 2 * (SEL_THREADS_HOST / 32);                   // one row pair per warp
    const int per_q = std::max(1, 148 / n_q);                            // CTAs per query
    const int bpc = std::max(PAIRS, ceil_div(ceil_div(n_blk, per_q), PAIRS) * PAIRS);
    const int score_ctas = ceil_div(n_blk, bpc);
    // the scores, then one ballot word per 32 candidates (and per selecting warp, its last round)
    const size_t sel_smem = (size_t) w.scores_stride * 4 + ((size_t) ceil_div(w.scores_stride, 32) + SEL_THREADS_HOST / 32) * 4;
    if (sel_smem > 160 * 1024) return QSA_ERR_UNSUPPORTED;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(score_ctas, n_q);
    cfg.blockDim = dim3(SEL_THREADS_HOST);
    cfg.dynamicSmemBytes = sel_smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;      // overlaps the append's tail
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = chained ? 1 : 0;
    return cuda_status(cudaLaunchKernelEx(&cfg, score_select_kernel, d, items, cache0.pool, n_past0, q_idx, bpc,
        reinterpret_cast<float *>(ws + w.scores), w.scores_stride, reinterpret_cast<unsigned *>(ws + w.cnt_sel),
        reinterpret_cast<int *>(ws + w.sel), reinterpret_cast<int *>(ws + w.nsel), sel_out, status, cand_scores));
}

// The states of a sharded step in one array (null: none, the output instead).
StateDst local_states(float * p) {
    StateDst s{};
    if (p) { s.base[0] = p; s.n = 1; }
    return s;
}

// Attention over the selection held in the workspace (and the merge of split queries).
qsa_status launch_attend(const DevDesc & d, const WsLayout & w, int n_q, const qsa_decode_item * items,
                         qsa_layer_cache cache0, int n_past0, const void * q, int q_type, OutSpec out,
                         unsigned char * ws, cudaStream_t st, bool chained, const StateDst & sdst = StateDst{}) {
    return cuda_status(launch_attn(d, st, chained, n_q, items, cache0, n_past0, q, q_type,
                                   reinterpret_cast<const int *>(ws + w.sel), reinterpret_cast<const int *>(ws + w.nsel),
                                   w.tiles_per_cta, w.max_chunks, reinterpret_cast<float *>(ws + w.part_o),
                                   reinterpret_cast<float *>(ws + w.part_ml), out,
                                   reinterpret_cast<uint32_t *>(ws + w.status), sdst));
}

}  // namespace

// Bytes at the start of a decode workspace that must be zero before a call: the status word and
// the arrival counters (the kernels leave their counters at zero, but the region's extent depends
// on the batch size).
size_t decode_workspace_zero_prefix(const qsa_desc * d, int32_t batch, int32_t max_n_kv) {
    return ws_layout(make_dev(d), batch, max_n_kv).scores;
}

DevDesc dev_desc(const qsa_desc * d) { return make_dev(d); }

}  // namespace qsa

using namespace qsa;

extern "C" {

const char * qsa_status_string(qsa_status s) {
    switch (s) {
        case QSA_OK: return "ok";
        case QSA_ERR_INVALID: return "invalid argument";
        case QSA_ERR_CUDA: return "CUDA error";
        case QSA_ERR_TIMEOUT: return "device wait timed out";
        case QSA_ERR_UNSUPPORTED: return "unsupported shape or type";
        case QSA_ERR_WORKSPACE: return "workspace too small";
        case QSA_ERR_DEVICE_ARG: return "out-of-range value found on the device";
    }
    return "unknown status";
}

qsa_status qsa_desc_check(const qsa_desc * d) {
    if (!d) return QSA_ERR_INVALID;
    if (d->n_head <= 0 || d->n_head_kv <= 0 || d->n_head % d->n_head_kv != 0) return QSA_ERR_INVALID;
    if (d->ratio <= 0 || d->n_ctx <= 0 || d->n_ctx % d->ratio != 0) return QSA_ERR_INVALID;
    if (d->top_k_blocks <= 0 || d->window < 0 || d->idx_n_head <= 0) return QSA_ERR_INVALID;
    if (d->rope_dim <= 0 || d->rope_dim % 2 != 0 || d->rope_dim > d->idx_dim) return QSA_ERR_INVALID;
    if (d->type_k != QSA_TYPE_Q8_0 && d->type_k != QSA_TYPE_F16) return QSA_ERR_INVALID;
    if (d->type_v != QSA_TYPE_Q8_0 && d->type_v != QSA_TYPE_F16) return QSA_ERR_INVALID;
    // what the kernels of this version are written for
    if (d->head_dim != HEAD_DIM) return QSA_ERR_UNSUPPORTED;
    if (d->n_head / d->n_head_kv > GQA_TILE || d->n_head_kv > 2) return QSA_ERR_UNSUPPORTED;
    if (d->idx_dim != MAX_IDX_DIM || d->idx_n_head > 4 || d->rope_dim % 8 != 0) return QSA_ERR_UNSUPPORTED;
    if (d->type_k != d->type_v) return QSA_ERR_UNSUPPORTED;
    if (d->top_k_blocks + n_force_of(d) > MAX_KB) return QSA_ERR_UNSUPPORTED;
    if (d->placement & ~(uint32_t) (QSA_KV_HOST | QSA_IDX_HOST)) return QSA_ERR_INVALID;
    if (d->ratio > 256) return QSA_ERR_UNSUPPORTED;        // a block of raw keys is staged in shared memory
    return QSA_OK;
}

int32_t qsa_k_blocks(const qsa_desc * d) { return d ? d->top_k_blocks + n_force_of(d) : 0; }

size_t qsa_row_bytes(const qsa_desc * d, int32_t which) {
    if (!d) return 0;
    const int64_t kv_dim = (int64_t) d->n_head_kv * d->head_dim;
    switch (which) {
        case 0: return kv_row_bytes(d->type_k, kv_dim);
        case 1: return kv_row_bytes(d->type_v, kv_dim);
        case 2: return (size_t) d->idx_dim * 2;
        case 3: return (size_t) d->idx_dim * 2;
        default: return 0;
    }
}

size_t qsa_cache_bytes(const qsa_desc * d, int32_t which) {
    if (!d) return 0;
    const size_t rows = which == 3 ? (size_t) (d->n_ctx / std::max(1, d->ratio)) : (size_t) d->n_ctx;
    return rows * qsa_row_bytes(d, which);
}

namespace {
qsa_status append_impl(const DevDesc & d, const qsa_layer_cache * cache, int32_t pos0, int32_t n_tok,
                       const float * k, const float * v, const float * kidx, qsa_stream_t stream) {
    if ((k && !cache->k) || (v && !cache->v) || (kidx && (!cache->idx || !cache->pool))) return QSA_ERR_INVALID;
    if (n_tok == 0) return QSA_OK;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    append_rows_kernel<<<n_tok, 256, 0, st>>>(d, *cache, pos0, k, v, kidx);
    if (kidx) {
        const int b0 = pos0 / d.ratio, b1 = (pos0 + n_tok) / d.ratio;   // blocks complete after the append
        if (b1 > b0) {
            const int n = b1 - b0;
            pool_blocks_kernel<<<ceil_div(n, 8), 256, 0, st>>>(d, cache->idx, cache->pool, b0, n, nullptr);
        }
    }
    return cuda_status(cudaGetLastError());
}
}  // namespace

qsa_status qsa_append(const qsa_desc * dd, const qsa_layer_cache * cache, int32_t pos0, int32_t n_tok,
                      const float * k, const float * v, const float * kidx, qsa_stream_t stream) {
    qsa_status s = qsa_desc_check(dd);
    if (s != QSA_OK) return s;
    if (!cache || pos0 < 0 || n_tok < 0 || (int64_t) pos0 + n_tok > dd->n_ctx) return QSA_ERR_INVALID;
    return append_impl(make_dev(dd), cache, pos0, n_tok, k, v, kidx, stream);
}

qsa_status qsa_shard_append(const qsa_desc * dd, const qsa_layer_cache * cache, int32_t blk_lo, int32_t blk_hi,
                            int32_t pos0, int32_t n_tok, const float * k, const float * v, const float * kidx,
                            qsa_stream_t stream) {
    qsa_status s = qsa_desc_check(dd);
    if (s != QSA_OK) return s;
    if (!cache || blk_lo < 0 || blk_hi <= blk_lo || (int64_t) blk_hi * dd->ratio > dd->n_ctx) return QSA_ERR_INVALID;
    if (n_tok < 0 || pos0 < blk_lo * dd->ratio || (int64_t) pos0 + n_tok > (int64_t) blk_hi * dd->ratio)
        return QSA_ERR_INVALID;
    DevDesc d = make_dev(dd);
    d.shard_blk0 = blk_lo;
    d.shard_blk1 = blk_hi;
    return append_impl(d, cache, pos0, n_tok, k, v, kidx, stream);
}

qsa_status qsa_pool_rebuild(const qsa_desc * dd, const qsa_layer_cache * cache, int32_t blk0, int32_t n_blk,
                            float * pooled_f32, qsa_stream_t stream) {
    qsa_status s = qsa_desc_check(dd);
    if (s != QSA_OK) return s;
    if (!cache || !cache->idx || !cache->pool || blk0 < 0 || n_blk < 0 ||
        (int64_t) (blk0 + n_blk) * dd->ratio > dd->n_ctx) return QSA_ERR_INVALID;
    if (n_blk == 0) return QSA_OK;
    const DevDesc d = make_dev(dd);
    pool_blocks_kernel<<<ceil_div(n_blk, 8), 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
        d, cache->idx, cache->pool, blk0, n_blk, pooled_f32);
    return cuda_status(cudaGetLastError());
}

size_t qsa_decode_workspace_size(const qsa_desc * dd, int32_t batch, int32_t max_n_kv) {
    if (qsa_desc_check(dd) != QSA_OK || batch <= 0 || max_n_kv <= 0) return 0;
    return ws_layout(make_dev(dd), batch, max_n_kv).total;
}

size_t qsa_shard_workspace_size(const qsa_desc * dd, int32_t batch, int32_t max_n_kv, int32_t blk_lo, int32_t blk_hi) {
    if (qsa_desc_check(dd) != QSA_OK || batch <= 0 || max_n_kv <= 0 || blk_lo < 0 || blk_hi <= blk_lo) return 0;
    DevDesc d = make_dev(dd);
    d.shard_blk0 = blk_lo;
    d.shard_blk1 = blk_hi;
    return ws_layout(d, batch, max_n_kv).total;
}

namespace {
// The prefill's KV-stationary attention applies (and how many blocks its buckets cover).
bool prefill_kv_path(const DevDesc & d, int T) { return T >= 64 && prefill_kv_supported(d, T); }
int prefill_n_blocks(const DevDesc & d, int max_n_kv) { return std::max(1, ceil_div(max_n_kv, d.ratio)); }
}  // namespace

size_t qsa_prefill_workspace_size(const qsa_desc * dd, int32_t T, int32_t max_n_kv) {
    const size_t base = qsa_decode_workspace_size(dd, T, max_n_kv);
    if (base == 0) return 0;
    const DevDesc d = make_dev(dd);
    return prefill_kv_path(d, T) ? base + prefill_kv_workspace(d, T, prefill_n_blocks(d, max_n_kv)) : base;
}

qsa_status qsa_workspace_init(void * ws, size_t ws_bytes, qsa_stream_t stream) {
    if (!ws || ws_bytes == 0) return QSA_ERR_WORKSPACE;
    return cuda_status(cudaMemsetAsync(ws, 0, ws_bytes, reinterpret_cast<cudaStream_t>(stream)));
}

namespace {
// The append of a decode step: a plain launch, never a programmatic dependent.  Everything
// before it in the stream (whatever wrote the items, q_idx and the new rows) is then complete
// when the chain starts, which the selection relies on: launched behind the append, it reads
// the items and q_idx before its own griddepcontrol.wait.
// The first kernel of its call, yet a programmatic launch: its launch overlaps the kernel ahead,
// and it waits for that kernel before it reads anything.  Waiting on the kernel ahead covers all
// earlier work in the stream, as that kernel completes only after its own predecessors (an
// ordinary launch starts after them; a programmatic one waits for them before it exits).
qsa_status launch_append_decode(const DevDesc & d, cudaStream_t st, int batch, const qsa_decode_item * items,
                                const float * k_new, const float * v_new, const float * kidx_new, uint32_t * status) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(batch);
    cfg.blockDim = dim3(APPEND_DECODE_THREADS);
    cfg.dynamicSmemBytes = append_decode_smem(d);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cuda_status(cudaLaunchKernelEx(&cfg, append_decode_kernel, d, items, k_new, v_new, kidx_new, status));
}

qsa_status decode_common(const qsa_desc * dd, const qsa_decode_item * items, int32_t batch, int32_t max_n_kv,
                         void * ws, size_t ws_bytes, DevDesc & d, WsLayout & w) {
    qsa_status s = qsa_desc_check(dd);
    if (s != QSA_OK) return s;
    if (!items || batch <= 0 || max_n_kv <= 0 || max_n_kv > dd->n_ctx) return QSA_ERR_INVALID;
    d = make_dev(dd);
    w = ws_layout(d, batch, max_n_kv);
    if (!ws || ws_bytes < w.total) return QSA_ERR_WORKSPACE;
    return set_attrs();
}
}  // namespace

qsa_status qsa_decode_append(const qsa_desc * dd, const qsa_decode_item * items, int32_t batch, int32_t max_n_kv,
                             const float * k_new, const float * v_new, const float * kidx_new,
                             void * ws, size_t ws_bytes, qsa_stream_t stream) {
    DevDesc d; WsLayout w;
    qsa_status s = decode_common(dd, items, batch, max_n_kv, ws, ws_bytes, d, w);
    if (s != QSA_OK) return s;
    if (!k_new || !v_new || !kidx_new) return QSA_ERR_INVALID;
    return launch_append_decode(d, reinterpret_cast<cudaStream_t>(stream), batch, items, k_new, v_new, kidx_new,
                                reinterpret_cast<uint32_t *>(static_cast<unsigned char *>(ws) + w.status));
}

qsa_status qsa_decode_select(const qsa_desc * dd, const qsa_decode_item * items, int32_t batch, int32_t max_n_kv,
                             const float * q_idx, int32_t * sel_out, void * ws, size_t ws_bytes, qsa_stream_t stream) {
    DevDesc d; WsLayout w;
    qsa_status s = decode_common(dd, items, batch, max_n_kv, ws, ws_bytes, d, w);
    if (s != QSA_OK) return s;
    if (!q_idx) return QSA_ERR_INVALID;
    qsa_layer_cache none{};
    return launch_select(d, w, batch, items, none, 0, q_idx, sel_out, static_cast<unsigned char *>(ws),
                         reinterpret_cast<cudaStream_t>(stream), false);
}

qsa_status qsa_decode_attend(const qsa_desc * dd, const qsa_decode_item * items, int32_t batch, int32_t max_n_kv,
                             const void * q, int32_t q_type, float * out, void * ws, size_t ws_bytes,
                             qsa_stream_t stream) {
    DevDesc d; WsLayout w;
    qsa_status s = decode_common(dd, items, batch, max_n_kv, ws, ws_bytes, d, w);
    if (s != QSA_OK) return s;
    if (!q || !out || (q_type != QSA_TYPE_BF16 && q_type != QSA_TYPE_F32)) return QSA_ERR_INVALID;
    qsa_layer_cache none{};
    return launch_attend(d, w, batch, items, none, 0, q, q_type, OutSpec{out, nullptr, nullptr, 0}, static_cast<unsigned char *>(ws),
                         reinterpret_cast<cudaStream_t>(stream), false);
}

namespace {
// An output descriptor from the public arguments: out and/or the gated product z (gate and z both
// given, z_type QSA_TYPE_BF16 or QSA_TYPE_F32, 8- or 16-byte aligned as its element type needs).
bool out_spec(float * out, const float * gate, void * z, int32_t z_type, OutSpec & o) {
    o = OutSpec{out, nullptr, nullptr, 0};
    if ((gate != nullptr) != (z != nullptr)) return false;
    if (z) {
        if (z_type != QSA_TYPE_BF16 && z_type != QSA_TYPE_F32) return false;
        if ((reinterpret_cast<uintptr_t>(gate) & 15u) || (reinterpret_cast<uintptr_t>(z) & (z_type == QSA_TYPE_BF16 ? 7u : 15u)))
            return false;
        o.gate = gate; o.z = z; o.z_bf16 = z_type == QSA_TYPE_BF16;
    }
    if (out && (reinterpret_cast<uintptr_t>(out) & 15u)) return false;
    return out || z;
}

qsa_status decode_impl(const qsa_desc * dd, const qsa_decode_item * items, int32_t batch, int32_t max_n_kv,
                       const void * q, int32_t q_type, const float * q_idx,
                       const float * k_new, const float * v_new, const float * kidx_new,
                       const OutSpec & out, int32_t * sel_out, void * ws, size_t ws_bytes, qsa_stream_t stream) {
    DevDesc d; WsLayout w;
    qsa_status s = decode_common(dd, items, batch, max_n_kv, ws, ws_bytes, d, w);
    if (s != QSA_OK) return s;
    if (!q || !q_idx || (q_type != QSA_TYPE_BF16 && q_type != QSA_TYPE_F32)) return QSA_ERR_INVALID;
    const bool any_new = k_new || v_new || kidx_new;
    if (any_new && !(k_new && v_new && kidx_new)) return QSA_ERR_INVALID;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    unsigned char * wsb = static_cast<unsigned char *>(ws);
    if (any_new)
        if ((s = launch_append_decode(d, st, batch, items, k_new, v_new, kidx_new,
                                      reinterpret_cast<uint32_t *>(wsb + w.status))) != QSA_OK) return s;
    qsa_layer_cache none{};
    if ((s = launch_select(d, w, batch, items, none, 0, q_idx, sel_out, wsb, st, any_new)) != QSA_OK) return s;
    return launch_attend(d, w, batch, items, none, 0, q, q_type, out, wsb, st, true);
}
}  // namespace

qsa_status qsa_decode(const qsa_desc * dd, const qsa_decode_item * items, int32_t batch, int32_t max_n_kv,
                      const void * q, int32_t q_type, const float * q_idx,
                      const float * k_new, const float * v_new, const float * kidx_new,
                      float * out, int32_t * sel_out, void * ws, size_t ws_bytes, qsa_stream_t stream) {
    if (!out) return QSA_ERR_INVALID;
    return decode_impl(dd, items, batch, max_n_kv, q, q_type, q_idx, k_new, v_new, kidx_new,
                       OutSpec{out, nullptr, nullptr, 0}, sel_out, ws, ws_bytes, stream);
}

qsa_status qsa_decode_gated(const qsa_desc * dd, const qsa_decode_item * items, int32_t batch, int32_t max_n_kv,
                            const void * q, int32_t q_type, const float * q_idx,
                            const float * k_new, const float * v_new, const float * kidx_new,
                            const float * gate, void * z, int32_t z_type, float * out,
                            int32_t * sel_out, void * ws, size_t ws_bytes, qsa_stream_t stream) {
    OutSpec o;
    if (!gate || !z || !out_spec(out, gate, z, z_type, o)) return QSA_ERR_INVALID;
    return decode_impl(dd, items, batch, max_n_kv, q, q_type, q_idx, k_new, v_new, kidx_new, o, sel_out, ws, ws_bytes,
                       stream);
}

namespace {
qsa_status prefill_impl(const qsa_desc * dd, const qsa_layer_cache * cache, int32_t n_past, int32_t T,
                        const void * q, int32_t q_type, const float * q_idx,
                        const float * k_new, const float * v_new, const float * kidx_new,
                        const OutSpec & out, int32_t * sel_out, void * ws, size_t ws_bytes, qsa_stream_t stream) {
    qsa_status s = qsa_desc_check(dd);
    if (s != QSA_OK) return s;
    if (!cache || n_past < 0 || T <= 0 || (int64_t) n_past + T > dd->n_ctx || !q || !q_idx) return QSA_ERR_INVALID;
    if (!cache->k || !cache->v || !cache->idx || !cache->pool) return QSA_ERR_INVALID;
    if (q_type != QSA_TYPE_BF16 && q_type != QSA_TYPE_F32) return QSA_ERR_INVALID;
    const bool any_new = k_new || v_new || kidx_new;
    if (any_new && !(k_new && v_new && kidx_new)) return QSA_ERR_INVALID;
    const DevDesc d = make_dev(dd);
    const WsLayout w = ws_layout(d, T, n_past + T);
    // the block-grouped path reads the caches with TMA, which wants 16-byte aligned rows
    const bool kv_path = prefill_kv_path(d, T) && !d.kv_host && reinterpret_cast<uintptr_t>(cache->k) % 16 == 0 &&
                         reinterpret_cast<uintptr_t>(cache->v) % 16 == 0;
    const size_t need = kv_path ? w.total + prefill_kv_workspace(d, T, prefill_n_blocks(d, n_past + T)) : w.total;
    if (!ws || ws_bytes < need) return QSA_ERR_WORKSPACE;
    if ((s = set_attrs()) != QSA_OK) return s;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    if (any_new) {
        if ((s = qsa_append(dd, cache, n_past, T, k_new, v_new, kidx_new, stream)) != QSA_OK) return s;
    }
    unsigned char * wsb = static_cast<unsigned char *>(ws);
    if (d.idx_n_head == 1 || d.idx_n_head == 2 || d.idx_n_head == 4) {
        // scores of every query of the chunk against every block whole at its end on the tensor
        // cores, then one warp per query selects
        uint32_t * status = reinterpret_cast<uint32_t *>(wsb + w.status);
        float * scores = reinterpret_cast<float *>(wsb + w.scores);
        cudaError_t e = launch_prefill_scores_tc(d, st, q_idx, T, cache->pool, (n_past + T) / d.ratio, scores,
                                                 w.scores_stride, status);
        if (e == cudaSuccess)
            e = launch_select_scores_warp(d, st, n_past, T, scores, w.scores_stride, reinterpret_cast<int *>(wsb + w.sel),
                                          reinterpret_cast<int *>(wsb + w.nsel), sel_out, status);
        if (e != cudaSuccess) return QSA_ERR_CUDA;
    } else if ((s = launch_select(d, w, T, nullptr, *cache, n_past, q_idx, sel_out, wsb, st, any_new)) != QSA_OK) {
        return s;
    }
    if (kv_path)
        return cuda_status(launch_prefill_attn_kv(d, st, *cache, n_past, T, q, q_type, reinterpret_cast<const int *>(wsb + w.sel),
                                                  reinterpret_cast<const int *>(wsb + w.nsel), prefill_n_blocks(d, n_past + T),
                                                  wsb + w.total, out, reinterpret_cast<uint32_t *>(wsb + w.status)));
    return launch_attend(d, w, T, nullptr, *cache, n_past, q, q_type, out, wsb, st, true);
}
}  // namespace

qsa_status qsa_prefill(const qsa_desc * dd, const qsa_layer_cache * cache, int32_t n_past, int32_t T,
                       const void * q, int32_t q_type, const float * q_idx,
                       const float * k_new, const float * v_new, const float * kidx_new,
                       float * out, int32_t * sel_out, void * ws, size_t ws_bytes, qsa_stream_t stream) {
    if (!out) return QSA_ERR_INVALID;
    return prefill_impl(dd, cache, n_past, T, q, q_type, q_idx, k_new, v_new, kidx_new, OutSpec{out, nullptr, nullptr, 0},
                        sel_out, ws, ws_bytes, stream);
}

qsa_status qsa_prefill_gated(const qsa_desc * dd, const qsa_layer_cache * cache, int32_t n_past, int32_t T,
                             const void * q, int32_t q_type, const float * q_idx,
                             const float * k_new, const float * v_new, const float * kidx_new,
                             const float * gate, void * z, int32_t z_type, float * out,
                             int32_t * sel_out, void * ws, size_t ws_bytes, qsa_stream_t stream) {
    OutSpec o;
    if (!gate || !z || !out_spec(out, gate, z, z_type, o)) return QSA_ERR_INVALID;
    return prefill_impl(dd, cache, n_past, T, q, q_type, q_idx, k_new, v_new, kidx_new, o, sel_out, ws, ws_bytes, stream);
}

qsa_status qsa_check(void * ws, size_t ws_bytes, qsa_stream_t stream) {
    if (!ws || ws_bytes < 16) return QSA_ERR_WORKSPACE;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    uint32_t h = 0;
    cudaError_t e = cudaMemcpyAsync(&h, ws, 4, cudaMemcpyDeviceToHost, st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    if (e != cudaSuccess) return QSA_ERR_CUDA;
    if (h != 0) {
        if (cudaMemsetAsync(ws, 0, 4, st) != cudaSuccess || cudaStreamSynchronize(st) != cudaSuccess) return QSA_ERR_CUDA;
        if (h & DEV_TIMEOUT) return QSA_ERR_TIMEOUT;
        return QSA_ERR_DEVICE_ARG;
    }
    return QSA_OK;
}

// ---- KV-sequence-sharded decode
size_t qsa_shard_state_floats(const qsa_desc * d) {
    (void) d;
    return (size_t) attn_state_rows() * (2 + HEAD_DIM);
}

namespace {
qsa_status shard_common(const qsa_desc * dd, const qsa_decode_item * items, int32_t batch, int32_t max_n_kv,
                        int32_t blk_lo, int32_t blk_hi, void * ws, size_t ws_bytes, DevDesc & d, WsLayout & w) {
    qsa_status s = qsa_desc_check(dd);
    if (s != QSA_OK) return s;
    if (!items || batch <= 0 || max_n_kv <= 0 || max_n_kv > dd->n_ctx) return QSA_ERR_INVALID;
    if (blk_lo < 0 || blk_hi <= blk_lo || (int64_t) blk_hi * dd->ratio > dd->n_ctx) return QSA_ERR_INVALID;
    d = make_dev(dd);
    d.shard_blk0 = blk_lo;
    d.shard_blk1 = blk_hi;
    w = ws_layout(d, batch, max_n_kv);
    if (!ws || ws_bytes < w.total) return QSA_ERR_WORKSPACE;
    return set_attrs();
}
}  // namespace

qsa_status qsa_shard_candidates(const qsa_desc * dd, const qsa_decode_item * items, int32_t batch, int32_t max_n_kv,
                                int32_t blk_lo, int32_t blk_hi, const float * q_idx,
                                const float * k_new, const float * v_new, const float * kidx_new,
                                int32_t * cand, void * ws, size_t ws_bytes, qsa_stream_t stream) {
    DevDesc d; WsLayout w;
    qsa_status s = shard_common(dd, items, batch, max_n_kv, blk_lo, blk_hi, ws, ws_bytes, d, w);
    if (s != QSA_OK) return s;
    if (!q_idx || !cand) return QSA_ERR_INVALID;
    const bool any_new = k_new || v_new || kidx_new;
    if (any_new && !(k_new && v_new && kidx_new)) return QSA_ERR_INVALID;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    unsigned char * wsb = static_cast<unsigned char *>(ws);
    if (any_new)           // only the shard holding a query's cell writes it (the kernel skips the rest)
        if ((s = launch_append_decode(d, st, batch, items, k_new, v_new, kidx_new,
                                      reinterpret_cast<uint32_t *>(wsb + w.status))) != QSA_OK) return s;
    qsa_layer_cache none{};
    return launch_select(d, w, batch, items, none, 0, q_idx, cand, wsb, st, any_new,
                         reinterpret_cast<float *>(cand + (size_t) batch * d.kb));
}

qsa_status qsa_shard_attend(const qsa_desc * dd, const qsa_decode_item * items, int32_t batch, int32_t max_n_kv,
                            int32_t blk_lo, int32_t blk_hi, int32_t n_shards, const int32_t * all_cand,
                            int32_t cand_stride, const void * q, int32_t q_type, float * state,
                            int32_t * sel_out, void * ws, size_t ws_bytes, qsa_stream_t stream) {
    DevDesc d; WsLayout w;
    qsa_status s = shard_common(dd, items, batch, max_n_kv, blk_lo, blk_hi, ws, ws_bytes, d, w);
    if (s != QSA_OK) return s;
    if (n_shards <= 0 || !all_cand || !q || !state) return QSA_ERR_INVALID;
    if (q_type != QSA_TYPE_BF16 && q_type != QSA_TYPE_F32) return QSA_ERR_INVALID;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    unsigned char * wsb = static_cast<unsigned char *>(ws);
    const size_t stride = cand_stride > 0 ? (size_t) cand_stride : (size_t) 2 * batch * d.kb;
    if (stride < (size_t) 2 * batch * d.kb) return QSA_ERR_INVALID;
    cudaError_t e = launch_shard_select(d, st, items, n_shards, batch, all_cand, stride, blk_lo, blk_hi, sel_out, reinterpret_cast<int *>(wsb + w.sel), reinterpret_cast<int *>(wsb + w.nsel),
                                        reinterpret_cast<uint32_t *>(wsb + w.status));
    if (e == cudaErrorInvalidValue) return QSA_ERR_UNSUPPORTED;       // too many candidates for one CTA
    if (e != cudaSuccess) return QSA_ERR_CUDA;
    qsa_layer_cache none{};
    return launch_attend(d, w, batch, items, none, 0, q, q_type, OutSpec{nullptr, nullptr, nullptr, 0}, wsb, st, true,
                         local_states(state));
}

// ---- KV-sharded decode with the indexer caches replicated on every rank
qsa_status qsa_shard_append_ri(const qsa_desc * dd, const qsa_layer_cache * cache, int32_t blk_lo, int32_t blk_hi,
                               int32_t pos0, int32_t n_tok, const float * k, const float * v, const float * kidx,
                               qsa_stream_t stream) {
    qsa_status s = qsa_desc_check(dd);
    if (s != QSA_OK) return s;
    if (!cache || blk_lo < 0 || blk_hi <= blk_lo || (int64_t) blk_hi * dd->ratio > dd->n_ctx) return QSA_ERR_INVALID;
    if (pos0 < 0 || n_tok < 0 || (int64_t) pos0 + n_tok > dd->n_ctx) return QSA_ERR_INVALID;
    DevDesc d = make_dev(dd);
    d.shard_blk0 = blk_lo;
    d.shard_blk1 = blk_hi;
    d.shard_ri = 1;
    return append_impl(d, cache, pos0, n_tok, k, v, kidx, stream);
}

qsa_status qsa_shard_decode_ri(const qsa_desc * dd, const qsa_decode_item * items, int32_t batch, int32_t max_n_kv,
                               int32_t blk_lo, int32_t blk_hi, const void * q, int32_t q_type, const float * q_idx,
                               const float * k_new, const float * v_new, const float * kidx_new, float * state,
                               int32_t * sel_out, void * ws, size_t ws_bytes, qsa_stream_t stream) {
    DevDesc d; WsLayout w;
    qsa_status s = shard_common(dd, items, batch, max_n_kv, blk_lo, blk_hi, ws, ws_bytes, d, w);
    if (s != QSA_OK) return s;
    d.shard_ri = 1;
    if (!q || !q_idx || !state || (q_type != QSA_TYPE_BF16 && q_type != QSA_TYPE_F32)) return QSA_ERR_INVALID;
    const bool any_new = k_new || v_new || kidx_new;
    if (any_new && !(k_new && v_new && kidx_new)) return QSA_ERR_INVALID;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    unsigned char * wsb = static_cast<unsigned char *>(ws);
    if (any_new)           // every rank writes the raw and pooled keys, the owning shard the K/V row
        if ((s = launch_append_decode(d, st, batch, items, k_new, v_new, kidx_new,
                                      reinterpret_cast<uint32_t *>(wsb + w.status))) != QSA_OK) return s;
    qsa_layer_cache none{};
    if ((s = launch_select(d, w, batch, items, none, 0, q_idx, sel_out, wsb, st, any_new)) != QSA_OK) return s;
    return launch_attend(d, w, batch, items, none, 0, q, q_type, OutSpec{nullptr, nullptr, nullptr, 0}, wsb, st, true,
                         local_states(state));
}

// ---- the replicated-index step with its state exchange fused into the kernels
namespace {
// This rank's slot and flag in every region of the channel, for `batch` states.
bool peer_targets(const qsa_peer_slots * ps, int batch, StateDst & sd, uint32_t * flag[MAX_STATE_DST],
                  size_t & stride) {
    if (!ps || ps->n_ranks <= 0 || ps->n_ranks > MAX_STATE_DST || ps->rank < 0 || ps->rank >= ps->n_ranks || !ps->epoch)
        return false;
    stride = ((size_t) batch * attn_state_rows() * (2 + HEAD_DIM) * 4 + 15) & ~(size_t) 15;
    sd = StateDst{};
    for (int p = 0; p < ps->n_ranks; p++) {
        unsigned char * r = static_cast<unsigned char *>(ps->region[p]);
        if (!r || reinterpret_cast<uintptr_t>(r) % 16 != 0) return false;
        sd.base[p] = reinterpret_cast<float *>(r + (size_t) ps->rank * stride);
        flag[p] = reinterpret_cast<uint32_t *>(r + (size_t) ps->n_ranks * stride) + ps->rank;
    }
    sd.n = ps->n_ranks;
    return true;
}
}  // namespace

qsa_status qsa_shard_decode_ri_peer(const qsa_desc * dd, const qsa_decode_item * items, int32_t batch, int32_t max_n_kv,
                                    int32_t blk_lo, int32_t blk_hi, const void * q, int32_t q_type, const float * q_idx,
                                    const float * k_new, const float * v_new, const float * kidx_new,
                                    const qsa_peer_slots * slots, int32_t * sel_out, void * ws, size_t ws_bytes,
                                    qsa_stream_t stream) {
    StateDst sd;
    uint32_t * flag[MAX_STATE_DST];
    size_t stride = 0;
    if (batch <= 0 || !peer_targets(slots, batch, sd, flag, stride)) return QSA_ERR_INVALID;
    if (!q || !q_idx || (q_type != QSA_TYPE_BF16 && q_type != QSA_TYPE_F32)) return QSA_ERR_INVALID;
    DevDesc d; WsLayout w;
    qsa_status s = shard_common(dd, items, batch, max_n_kv, blk_lo, blk_hi, ws, ws_bytes, d, w);
    if (s != QSA_OK) return s;
    d.shard_ri = 1;
    const bool any_new = k_new || v_new || kidx_new;
    if (any_new && !(k_new && v_new && kidx_new)) return QSA_ERR_INVALID;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    unsigned char * wsb = static_cast<unsigned char *>(ws);
    if (any_new)
        if ((s = launch_append_decode(d, st, batch, items, k_new, v_new, kidx_new,
                                      reinterpret_cast<uint32_t *>(wsb + w.status))) != QSA_OK) return s;
    qsa_layer_cache none{};
    if ((s = launch_select(d, w, batch, items, none, 0, q_idx, sel_out, wsb, st, any_new)) != QSA_OK) return s;
    if ((s = launch_attend(d, w, batch, items, none, 0, q, q_type, OutSpec{nullptr, nullptr, nullptr, 0}, wsb, st, true,
                           sd)) != QSA_OK) return s;
    return cuda_status(launch_peer_publish(st, flag, slots->n_ranks, slots->epoch));
}

qsa_status qsa_merge_states_peer(const qsa_desc * dd, const qsa_peer_slots * slots, int32_t batch, float * out,
                                 void * ws, size_t ws_bytes, qsa_stream_t stream) {
    qsa_status s = qsa_desc_check(dd);
    if (s != QSA_OK) return s;
    StateDst sd;
    uint32_t * flag[MAX_STATE_DST];
    size_t stride = 0;
    if (batch <= 0 || !out || !peer_targets(slots, batch, sd, flag, stride)) return QSA_ERR_INVALID;
    if (!ws || ws_bytes < 16) return QSA_ERR_WORKSPACE;
    const unsigned char * local = static_cast<const unsigned char *>(slots->region[slots->rank]);
    return cuda_status(launch_merge_states(make_dev(dd), reinterpret_cast<cudaStream_t>(stream), slots->n_ranks, batch,
                                           reinterpret_cast<const float *>(local),
                                           out, reinterpret_cast<const uint32_t *>(local + (size_t) slots->n_ranks * stride),
                                           slots->epoch, static_cast<uint32_t *>(ws)));
}

qsa_status qsa_merge_states(const qsa_desc * dd, int32_t n_parts, int32_t batch, const float * states, float * out,
                            qsa_stream_t stream) {
    qsa_status s = qsa_desc_check(dd);
    if (s != QSA_OK) return s;
    if (n_parts <= 0 || batch <= 0 || !states || !out) return QSA_ERR_INVALID;
    return cuda_status(launch_merge_states(make_dev(dd), reinterpret_cast<cudaStream_t>(stream), n_parts, batch,
                                           states, out));
}

int32_t qsa_version(void) { return 100; }

}  // extern "C"
