// qsa_attn.cu -- block-sparse split-K flash attention over the selected q8_0 / f16 KV rows.
//
// Reference: ggml_flash_attn_ext over the gathered cells with the cell mask, precision F32,
// scale 1/sqrt(head_dim), GQA (src/qwfn_graph.cpp:497-502, 530-541; prefill :362-403).
//
// Work item = (query t, chunk of 32-cell tiles), both KV heads in one CTA: 8 consumer warps and
// one producer warp, two CTAs per SM.  The selected blocks of a query, ascending, expand to a cell
// list (block b -> cells b*r .. b*r+r-1); a tile is 32 consecutive entries.
//   - the rows of one block are contiguous in the cache (row = both heads, 544 B in q8_0), so a
//     tile arrives as one bulk-async copy per block-run of valid rows (cells <= the query
//     position) for K and for V, into a ring of shared-memory stages completed by mbarrier
//     transaction counts; rows past the query or past the list are not fetched, they are masked
//     in registers (their scores -inf, their V scales / f16 values zero);
//   - the producer warp issues the copies of a stage once the consumers released it; consumer
//     warps 0-3 take KV head 0, warps 4-7 KV head 1; a warp pair owns 16 cells and splits the
//     256 dims in halves: each half-warp pair member computes a partial S over its 128 dims,
//     the pair exchanges them through shared memory, and each then accumulates O for its own
//     128 dims; the 8 query heads of a KV head are the N=8 dimension of mma.m16n8k16:
//     S^T = K Q^T (cells x heads), O^T += V^T P;
//   - q8_0 is dequantised in registers: int8 bytes become exact f16 integers; the K scale
//     multiplies the f32 partial dot of each 32-dim group, the V scale multiplies P;
//   - online softmax in the exp2 domain with warp shuffles; the two cell halves of a KV head
//     merge in shared memory; a query split over several CTAs leaves one unnormalised partial per CTA in
//     the workspace, merged by attn_merge_kernel, or attn_merge_small_kernel when no query has more
//     than 8 partials (launched programmatically behind the attention grid, they wait for it with
//     griddepcontrol.wait);
//   - sharded decode: the result is the unnormalised state (M, L, O) instead of the output, stored
//     to every destination of a StateDst (this rank's workspace, or its slot in every rank's
//     gather region over NVLink, published afterwards by peer_publish_kernel).
#include "qsa_kernels.cuh"

namespace qsa {

constexpr int ATT_CELLS   = 32;        // cells per tile (one pipeline stage)
constexpr int ATT_CWARPS  = 8;         // consumer warps: (KV head, 16-cell half, 128-dim half)
constexpr int ATT_THREADS = 32 * (ATT_CWARPS + 1);   // + the producer warp
constexpr int HROWS       = 16;        // 2 KV heads x 8 query heads: rows of the CTA state
constexpr int MERGE_THREADS = 256;     // attn_merge_kernel: threads per CTA

template <int KV_TYPE> struct AttnCfg;
template <> struct AttnCfg<QSA_TYPE_Q8_0> {
    static constexpr int HB       = 272;   // one head of a q8_0 row: 8 blocks x 34 B
    static constexpr int NSTAGE   = 3;     // 3 x 34.8 KB stages: two CTAs fit one SM's 228 KB
    static constexpr int MIN_CTAS = 2;     // CTAs per SM
};
template <> struct AttnCfg<QSA_TYPE_F16> {
    static constexpr int HB       = 512;
    static constexpr int NSTAGE   = 2;
    static constexpr int MIN_CTAS = 1;
};

// shared-memory row = the KV heads of the CTA (all heads of a row: n_head_kv <= 2)
template <int KV_TYPE> constexpr int attn_row_bytes() { return 2 * AttnCfg<KV_TYPE>::HB; }
template <int KV_TYPE> constexpr int attn_stage_bytes() { return 2 * ATT_CELLS * attn_row_bytes<KV_TYPE>(); }
// S exchange between the two dim-half warps of a pair: [2 tiles][consumer warps][32 lanes] float4
constexpr int ATT_XCH_BYTES = 2 * ATT_CWARPS * 32 * 16;
// Dynamic shared memory: the stage ring (the staged Q lives in stage 0 before the first tile),
// the S exchange, then the selected block list (kb entries).
template <int KV_TYPE> constexpr int attn_smem_bytes(int kb) {
    return AttnCfg<KV_TYPE>::NSTAGE * attn_stage_bytes<KV_TYPE>() + ATT_XCH_BYTES + ((kb * 4 + 15) & ~15);
}
// two q8_0 CTAs per SM (228 KB, 1 KB reserved per CTA) for up to 256 kept blocks
static_assert(AttnCfg<QSA_TYPE_Q8_0>::MIN_CTAS * (attn_smem_bytes<QSA_TYPE_Q8_0>(256) + 1024 + 128) <= 228 * 1024,
              "q8_0 attention CTAs per SM");
static_assert(HROWS * HEAD_DIM * 2 <= 2 * ATT_CELLS * 2 * AttnCfg<QSA_TYPE_Q8_0>::HB, "staged Q fits stage 0");
// the post-loop merge scratch (per-warp O, m, l) lives in the stage memory
static_assert(ATT_CWARPS * 8 * (HEAD_DIM / 2) * 4 + 3 * ATT_CWARPS * 8 * 4 + 2 * HROWS * 4 <=
              AttnCfg<QSA_TYPE_Q8_0>::NSTAGE * 2 * ATT_CELLS * 2 * AttnCfg<QSA_TYPE_Q8_0>::HB, "merge scratch");

__device__ __forceinline__ void ldmatrix_x4_trans(uint32_t (&a)[4], const void * p) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(a[0]), "=r"(a[1]), "=r"(a[2]), "=r"(a[3]) : "r"(smem_u32(p)));
}
__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
// Barrier of the `n` threads (whole warps) that name barrier `id` (1..15; 0 is __syncthreads).
__device__ __forceinline__ void named_bar_sync(int id, int n) {
    asm volatile("bar.sync %0, %1;" :: "r"(id), "r"(n) : "memory");
}

// 2^x with the hardware approximation (relative error below 2^-22; -inf gives 0): the softmax
// weights of the streaming loop.
__device__ __forceinline__ float ex2_fast(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// Cell of list entry `idx` of a query (cells of the selected blocks, in order).
__device__ __forceinline__ int list_cell(const int * sel, int r, int idx) { return sel[idx / r] * r + idx % r; }

// Tiles and chunks of a query with `nsel` selected blocks (the same in both kernels).
__device__ __forceinline__ int attn_n_chunks(const DevDesc & d, int nsel, int tiles_per_cta) {
    const int n_tiles = (nsel * d.ratio + ATT_CELLS - 1) / ATT_CELLS;
    return (n_tiles + tiles_per_cta - 1) / tiles_per_cta;
}

template <int KV_TYPE, int NKV>
__global__ void __launch_bounds__(ATT_THREADS, AttnCfg<KV_TYPE>::MIN_CTAS) attn_kernel(
        DevDesc d, const qsa_decode_item * __restrict__ items, qsa_layer_cache cache0, int n_past0,
        const void * __restrict__ q, int q_type,
        const int * sel_ws, const int * nsel_ws, int tiles_per_cta, int max_chunks,
        float * __restrict__ part_o, float * __restrict__ part_ml,
        OutSpec outs, uint32_t * __restrict__ status, StateDst sdst) {
    using Cfg = AttnCfg<KV_TYPE>;
    constexpr int NS = Cfg::NSTAGE, HB = Cfg::HB, RB = attn_row_bytes<KV_TYPE>();
    extern __shared__ __align__(128) unsigned char smem[];
    __shared__ uint64_t full_bar[NS];
    __shared__ uint64_t empty_bar[NS];
    __shared__ uint32_t vmask[NS];
    __shared__ int abort_wait;

    pdl_trigger();                             // the merge kernel may start; it waits for this grid
    const int t = blockIdx.y, chunk = blockIdx.x;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int r8 = lane >> 2, j4 = lane & 3;
    const int hs = (warp >> 2) & 1;           // consumer warp: KV head,
    const int cw = (warp >> 1) & 1;           //   16-cell half of the tile,
    const int dh = warp & 1;                  //   128-dim half (q8_0 groups 4dh..4dh+3)
    const bool producer = warp == ATT_CWARPS;
    const bool head_live = !producer && hs < NKV;
    __half * qs = reinterpret_cast<__half *>(smem);      // staged Q, then Q fragments (stage 0, before tile 0)
    float4 * xch = reinterpret_cast<float4 *>(smem + NS * attn_stage_bytes<KV_TYPE>());
    int * sel = reinterpret_cast<int *>(smem + NS * attn_stage_bytes<KV_TYPE>() + ATT_XCH_BYTES);

    // ---- prologue: every input load is independent, issued together
    int qpos;
    const uint8_t * kbase;
    const uint8_t * vbase;
    if (items) {
        qpos = items[t].n_past;
        kbase = (const uint8_t *) items[t].cache.k;
        vbase = (const uint8_t *) items[t].cache.v;
    } else {
        qpos = n_past0 + t;
        kbase = (const uint8_t *) cache0.k;
        vbase = (const uint8_t *) cache0.v;
    }
    if (d.shard_blk0 != 0) {                   // address of global cell 0 (only shard cells are read)
        const int64_t row0 = (int64_t) d.shard_blk0 * d.ratio;
        kbase = shard_row(kbase, row0, 0, d.rb_k);
        vbase = shard_row(vbase, row0, 0, d.rb_v);
    }
    {   // Q of the CTA's query heads -> f16 (the reference converts Q to K's vec_dot type, F16)
        for (int i = tid; i < HROWS * HEAD_DIM / 8; i += ATT_THREADS) {
            const int hrow = (i * 8) / HEAD_DIM, h = hrow & 7, g = hrow >> 3;
            float f[8];
            if (g < d.n_head_kv && h < d.gqa) {
                const size_t o = ((size_t) t * d.n_head + g * d.gqa + h) * HEAD_DIM + (i * 8) % HEAD_DIM;
                if (q_type == QSA_TYPE_BF16) {
                    const uint4 w = *reinterpret_cast<const uint4 *>(reinterpret_cast<const __nv_bfloat16 *>(q) + o);
                    const uint32_t ww[4] = {w.x, w.y, w.z, w.w};
                    #pragma unroll
                    for (int k = 0; k < 4; k++) {
                        f[2 * k]     = __uint_as_float(ww[k] << 16);
                        f[2 * k + 1] = __uint_as_float(ww[k] & 0xffff0000u);
                    }
                } else {
                    const float4 a = *reinterpret_cast<const float4 *>(reinterpret_cast<const float *>(q) + o);
                    const float4 b = *reinterpret_cast<const float4 *>(reinterpret_cast<const float *>(q) + o + 4);
                    f[0] = a.x; f[1] = a.y; f[2] = a.z; f[3] = a.w; f[4] = b.x; f[5] = b.y; f[6] = b.z; f[7] = b.w;
                }
            } else {
                #pragma unroll
                for (int k = 0; k < 8; k++) f[k] = 0.0f;
            }
            uint4 o4;
            o4.x = pack_f16x2(f[0], f[1]); o4.y = pack_f16x2(f[2], f[3]);
            o4.z = pack_f16x2(f[4], f[5]); o4.w = pack_f16x2(f[6], f[7]);
            *reinterpret_cast<uint4 *>(qs + i * 8) = o4;
        }
    }
    if (tid == 0) {
        for (int s = 0; s < NS; s++) {
            mbar_init(&full_bar[s], 1);
            mbar_init(&empty_bar[s], ATT_CWARPS);
        }
        abort_wait = 0;
        fence_mbar_init();
    }
    __syncthreads();                                  // staged Q and the barriers are visible
    // Q fragments (mma B operand) of each KV head, packed in lane order into shared memory (over
    // the staged Q, which only these two builders read): head n = r8 of the 8-head tile.
    uint32_t qf[16][2];
    const bool qbuilder = warp == 0 || warp == 4;
    if (qbuilder) {
        const __half * qrow = qs + (hs * 8 + r8) * HEAD_DIM;
        auto pk2 = [&](int d0, int d1) -> uint32_t {
            __half2 h = __halves2half2(qrow[d0], qrow[d1]);
            return *reinterpret_cast<uint32_t *>(&h);
        };
        if (KV_TYPE == QSA_TYPE_Q8_0) {
            // group g8 (32 dims), k-tile kt: virtual k (2j,2j+1) -> dims 8j+4kt+{0,2}; (2j+8,2j+9) -> 8j+4kt+{1,3}
            #pragma unroll
            for (int g8 = 0; g8 < 8; g8++)
                #pragma unroll
                for (int kt = 0; kt < 2; kt++) {
                    const int base = 32 * g8 + 8 * j4 + 4 * kt;
                    qf[2 * g8 + kt][0] = pk2(base + 0, base + 2);
                    qf[2 * g8 + kt][1] = pk2(base + 1, base + 3);
                }
        } else {
            #pragma unroll
            for (int kt = 0; kt < 16; kt++) {
                const int base = 16 * kt + 2 * j4;
                qf[kt][0] = pk2(base + 0, base + 1);
                qf[kt][1] = pk2(base + 8, base + 9);
            }
        }
    }
    __syncthreads();
    uint2 * qfrag = reinterpret_cast<uint2 *>(qs);       // [2 heads][16 k-steps][32 lanes]
    if (qbuilder) {
        #pragma unroll
        for (int k = 0; k < 16; k++) qfrag[(hs * 16 + k) * 32 + lane] = make_uint2(qf[k][0], qf[k][1]);
    }
    __syncthreads();
    // each consumer warp's Q fragments (its 8 k-steps of 16 dims) stay in registers for the whole
    // loop; afterwards stage 0 (where Q was staged) is free for tile 0
    uint2 qreg[8];
    if (!producer) {
        #pragma unroll
        for (int k = 0; k < 8; k++) qreg[k] = qfrag[(hs * 16 + 8 * dh + k) * 32 + lane];
    }
    __syncthreads();
    // Everything above depends on Q only, so it runs while the selection of this step is still in
    // progress (this grid is launched programmatically behind it).
    pdl_wait();                                // the selection of this step is complete
    const int nsel_raw = ld_dep(nsel_ws + t);
    // the producer requests the first entries of the list together with its length (one round
    // trip instead of two; entries past the length are never used)
    constexpr int SEL_PRE = 4;
    int sel_pre[SEL_PRE];
    if (producer) {
        #pragma unroll
        for (int k = 0; k < SEL_PRE; k++) {
            const int i = lane + 32 * k;
            sel_pre[k] = i < d.kb ? ld_dep(sel_ws + (size_t) t * d.kb + i) : -1;
        }
    }
    const bool pos_ok = qpos >= 0 && qpos < d.n_ctx;
    const int nsel = pos_ok ? max(0, min(nsel_raw, d.kb)) : 0;
    const int r = d.ratio;
    constexpr int RBr = NKV * HB;                        // cache row bytes: the run copies' row pitch
    const int n_cells = nsel * r;
    const int n_tiles = (n_cells + ATT_CELLS - 1) / ATT_CELLS;
    const int n_chunks = attn_n_chunks(d, nsel, tiles_per_cta);
    const size_t outq = (size_t) t * d.n_head * HEAD_DIM;     // element offset of query t's output
    // sharded mode: the unnormalised state [M 16][L 16][O 16x256] of query t instead of the output
    const bool stq = sdst.n > 0;
    const size_t sq0 = (size_t) t * (2 * HROWS + HROWS * HEAD_DIM);      // its offset in the state arrays
    if (n_chunks == 0) {                       // nothing selected (or a bad position): zero output
        if (chunk == 0) {
            if (stq) {
                for (int i = tid; i < 2 * HROWS + HROWS * HEAD_DIM; i += ATT_THREADS)
                    state_put(sdst, sq0 + i, i < HROWS ? -INFINITY : 0.0f);
            } else
                for (int i = 4 * tid; i < d.n_head * HEAD_DIM; i += 4 * ATT_THREADS)
                    out_store4(outs, outq + i, make_float4(0.f, 0.f, 0.f, 0.f));
        }
        return;
    }
    if (chunk >= n_chunks) return;             // the grid covers the longest query of the batch
    if ((smem_u32(smem) & 15u) != 0) {        // bulk copies need 16-byte aligned destinations
        if (tid == 0) set_status(status, DEV_BAD_SEL);
        return;
    }
    const int tile0 = chunk * tiles_per_cta;
    const int n_local = min(tiles_per_cta, n_tiles - tile0);

    auto stage_k = [&](int s) { return smem + s * attn_stage_bytes<KV_TYPE>(); };
    auto stage_v = [&](int s) { return smem + s * attn_stage_bytes<KV_TYPE>() + ATT_CELLS * RB; };  // RB >= row bytes
    // A bounded wait; after one wait of the CTA ran out, the others return at once (the status
    // word already says QSA_ERR_TIMEOUT; the results of this call are not used).
    auto wait_bar = [&](uint64_t * bar, uint32_t parity) -> bool {
        if (*reinterpret_cast<volatile int *>(&abort_wait)) return false;
        if (mbar_wait_bounded(bar, parity, status)) return true;
        *reinterpret_cast<volatile int *>(&abort_wait) = 1;
        return false;
    };

    float o[8][4];                                       // this warp's 128 dims x 8 heads
    #pragma unroll
    for (int i = 0; i < 8; i++) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.0f;
    // running reference maxima of the thread's two heads (log2 domain; finite start, so that a
    // weight 2^(s - m) never needs a guard), and the sums of weights
    float m0 = -1e30f, m1 = -1e30f, l0 = 0.0f, l1 = 0.0f;

    if (producer) {
        // only the producer reads the selected list: its lanes copy it (no CTA barrier)
        #pragma unroll
        for (int k = 0; k < SEL_PRE; k++)
            if (lane + 32 * k < nsel) sel[lane + 32 * k] = sel_pre[k];
        for (int i = lane + 32 * SEL_PRE; i < nsel; i += 32) sel[i] = ld_dep(sel_ws + (size_t) t * d.kb + i);
        __syncwarp();
        // Tile i goes to stage i % NS: one copy per block-run of valid rows (cells <= the query
        // position) for K and V, and the tile's 32-bit row-validity mask (written before the
        // release of the arrive).  Lane = tile entry.
        for (int i = 0; i < n_local; i++) {
            const int s = i % NS;
            if (i >= NS) {
                if (!wait_bar(&empty_bar[s], (uint32_t) (((i / NS) - 1) & 1))) break;
                fence_proxy_async_smem();
            }
            const int e_lo = (tile0 + i) * ATT_CELLS;
            const int e_hi = min(e_lo + ATT_CELLS, n_cells);
            const int j_lo = e_lo / r, j_hi = (e_hi - 1) / r;
            uint32_t bytes = 0;
            for (int j = j_lo + lane; j <= j_hi; j += 32) {
                const int a = max(e_lo, j * r), b = min(e_hi, (j + 1) * r);
                const int cs = sel[j] * r + (a - j * r);
                const int nv = max(0, min(b - a, qpos - cs + 1));
                bytes += (uint32_t) nv * RBr * 2;
            }
            #pragma unroll
            for (int off = 16; off > 0; off >>= 1) bytes += __shfl_xor_sync(0xffffffffu, bytes, off);
            const int ea = e_lo + lane;
            // r a multiple of the tile: the whole tile lies in block j_lo (no per-lane division)
            const int cell = (r % ATT_CELLS == 0) ? sel[j_lo] * r + (e_lo - j_lo * r) + lane : list_cell(sel, r, ea);
            const unsigned vm = __ballot_sync(0xffffffffu, ea < n_cells && cell <= qpos);
            if (d.kv_host) {
                // K and V in pinned host memory: the warp copies each run's rows with ordinary 16-byte
                // loads (bulk copies are not used on host memory), then one release arrive completes
                // the stage
                for (int j = j_lo; j <= j_hi; j++) {
                    const int a = max(e_lo, j * r), b = min(e_hi, (j + 1) * r);
                    const int cs = sel[j] * r + (a - j * r);
                    const int nv = max(0, min(b - a, qpos - cs + 1));
                    const int n16 = nv * RBr / 16;
                    const uint4 * sk = reinterpret_cast<const uint4 *>(kbase + (size_t) cs * d.rb_k);
                    const uint4 * sv = reinterpret_cast<const uint4 *>(vbase + (size_t) cs * d.rb_v);
                    uint4 * dk = reinterpret_cast<uint4 *>(stage_k(s) + (a - e_lo) * RBr);
                    uint4 * dv = reinterpret_cast<uint4 *>(stage_v(s) + (a - e_lo) * RBr);
                    for (int w = lane; w < n16; w += 64) {
                        const bool two = w + 32 < n16;
                        const uint4 k0 = sk[w], v0 = sv[w];
                        uint4 k1 = make_uint4(0u, 0u, 0u, 0u), v1 = k1;
                        if (two) { k1 = sk[w + 32]; v1 = sv[w + 32]; }
                        dk[w] = k0; dv[w] = v0;
                        if (two) { dk[w + 32] = k1; dv[w + 32] = v1; }
                    }
                }
                __syncwarp();
                if (lane == 0) {
                    vmask[s] = vm;
                    mbar_arrive(&full_bar[s]);
                }
                continue;
            }
            if (lane == 0) {
                vmask[s] = vm;
                mbar_arrive_expect_tx(&full_bar[s], bytes);
            }
            __syncwarp();
            for (int j = j_lo + lane; j <= j_hi; j += 32) {
                const int a = max(e_lo, j * r), b = min(e_hi, (j + 1) * r);
                const int cs = sel[j] * r + (a - j * r);
                const int nv = max(0, min(b - a, qpos - cs + 1));
                if (nv > 0) {
                    bulk_g2s(stage_k(s) + (a - e_lo) * RBr, kbase + (size_t) cs * d.rb_k, (uint32_t) nv * RBr, &full_bar[s]);
                    bulk_g2s(stage_v(s) + (a - e_lo) * RBr, vbase + (size_t) cs * d.rb_v, (uint32_t) nv * RBr, &full_bar[s]);
                }
            }
        }
    } else {
        const int rA = 16 * cw + r8, rB = rA + 8;           // this thread's S^T rows (cells of the tile)
        const int c0 = 16 * cw + 2 * j4;                     // this thread's V^T columns: c0+{0,1,8,9}
        const int hoff = hs * HB;                            // byte offset of this warp's head in a row
        constexpr int rb = NKV * HB;                         // row bytes (= smem row stride), K and V alike
        const int pair_bar = 1 + (warp >> 1);                // the two dim-half warps of (head, cells)
        const uint32_t negb[4] = {F16X2_NEG1152, F16X2_NEG1152, F16X2_NEG1152, F16X2_NEG1152};
        for (int i = 0; i < n_local; i++) {
            const int s = i % NS;
            const uint32_t ph = (uint32_t) ((i / NS) & 1);
            // every iteration reaches the pair barrier, also after a timed-out wait
            const bool ok = wait_bar(&full_bar[s], ph) && head_live;
            const uint32_t vm = vmask[s];
            const bool okA = (vm >> rA) & 1u, okB = (vm >> rB) & 1u;
            const uint8_t * Kt = stage_k(s) + hoff;
            const uint8_t * Vt = stage_v(s) + hoff;
            // ---- partial S^T = K Q^T over this warp's 128 dims, for its 16 cells x 8 heads
            float sc[4] = {0.f, 0.f, 0.f, 0.f};
            if (ok) {
                if (KV_TYPE == QSA_TYPE_Q8_0) {
                    // row bases are 4-byte aligned; q8_0 block g8 starts at byte 34*g8 (scale) + 2 (quants),
                    // so its quants are word aligned for odd g8 and 2 bytes off for even g8
                    const uint32_t * WA = reinterpret_cast<const uint32_t *>(Kt + rA * rb) + 34 * dh;
                    const uint32_t * WB = reinterpret_cast<const uint32_t *>(Kt + rB * rb) + 34 * dh;
                    const uint16_t * HA = reinterpret_cast<const uint16_t *>(WA);
                    const uint16_t * HB_ = reinterpret_cast<const uint16_t *>(WB);
                    #pragma unroll
                    for (int gg = 0; gg < 4; gg++) {            // group g8 = 4 dh + gg
                        uint32_t w0A, w1A, w0B, w1B;
                        if ((gg & 1) == 0) {
                            const int wi = 17 * (gg / 2) + 2 * j4;
                            const uint32_t a0 = WA[wi], a1 = WA[wi + 1], a2 = WA[wi + 2];
                            const uint32_t b0 = WB[wi], b1 = WB[wi + 1], b2 = WB[wi + 2];
                            w0A = __funnelshift_r(a0, a1, 16); w1A = __funnelshift_r(a1, a2, 16);
                            w0B = __funnelshift_r(b0, b1, 16); w1B = __funnelshift_r(b1, b2, 16);
                        } else {
                            const int wi = 17 * (gg / 2) + 9 + 2 * j4;
                            w0A = WA[wi]; w1A = WA[wi + 1];
                            w0B = WB[wi]; w1B = WB[wi + 1];
                        }
                        const float dA = f16_bits_to_f32(HA[17 * gg]);
                        const float dB = f16_bits_to_f32(HB_[17 * gg]);
                        const uint2 qa = qreg[2 * gg], qb2 = qreg[2 * gg + 1];
                        const uint32_t b0[2] = {qa.x, qa.y}, b1[2] = {qb2.x, qb2.y};
                        float c[4] = {0.f, 0.f, 0.f, 0.f};
                        // K + 1152 (exact f16 integers), then -1152 x the Q column sums
                        const uint32_t a0[4] = {i8x2_even_biased(w0A), i8x2_even_biased(w0B),
                                                i8x2_odd_biased(w0A), i8x2_odd_biased(w0B)};
                        const uint32_t a1[4] = {i8x2_even_biased(w1A), i8x2_even_biased(w1B),
                                                i8x2_odd_biased(w1A), i8x2_odd_biased(w1B)};
                        mma_f16_16816(c, negb, b0);
                        mma_f16_16816(c, negb, b1);
                        mma_f16_16816(c, a0, b0);
                        mma_f16_16816(c, a1, b1);
                        sc[0] = fmaf(dA, c[0], sc[0]); sc[1] = fmaf(dA, c[1], sc[1]);
                        sc[2] = fmaf(dB, c[2], sc[2]); sc[3] = fmaf(dB, c[3], sc[3]);
                    }
                } else {
                    #pragma unroll
                    for (int kk = 0; kk < 8; kk++) {
                        const int kt = 8 * dh + kk;
                        const uint8_t * ka = Kt + rA * rb + 2 * (16 * kt + 2 * j4);
                        const uint8_t * kb = Kt + rB * rb + 2 * (16 * kt + 2 * j4);
                        const uint32_t a[4] = {*reinterpret_cast<const uint32_t *>(ka), *reinterpret_cast<const uint32_t *>(kb),
                                               *reinterpret_cast<const uint32_t *>(ka + 16), *reinterpret_cast<const uint32_t *>(kb + 16)};
                        const uint2 qk = qreg[kk];
                        const uint32_t bq[2] = {qk.x, qk.y};
                        mma_f16_16816(sc, a, bq);
                    }
                }
            }
            // ---- the pair's two halves of S: exchange through shared memory (double-buffered by
            // tile parity, so one barrier per tile suffices); a + b == b + a, both warps agree
            if (head_live) {
                xch[((i & 1) * ATT_CWARPS + warp) * 32 + lane] = make_float4(sc[0], sc[1], sc[2], sc[3]);
                named_bar_sync(pair_bar, 64);
                const float4 pv = xch[((i & 1) * ATT_CWARPS + (warp ^ 1)) * 32 + lane];
                sc[0] += pv.x; sc[1] += pv.y; sc[2] += pv.z; sc[3] += pv.w;
            }
            if (ok) {
                // ---- mask, scale to the exp2 domain, online softmax (heads 2j, 2j+1 of this thread)
                sc[0] = okA ? sc[0] * d.scale_log2 : -INFINITY;
                sc[1] = okA ? sc[1] * d.scale_log2 : -INFINITY;
                sc[2] = okB ? sc[2] * d.scale_log2 : -INFINITY;
                sc[3] = okB ? sc[3] * d.scale_log2 : -INFINITY;
                float mx0 = fmaxf(sc[0], sc[2]), mx1 = fmaxf(sc[1], sc[3]);
                #pragma unroll
                for (int off = 4; off < 32; off <<= 1) {
                    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, off));
                    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, off));
                }
                // lazy rescale: the reference max moves only when a score exceeds it by more than 8
                // (weights stay below 2^8, well inside f16 and f32), so O and l are rescaled a few
                // times per query instead of at every new maximum
                const bool up0 = mx0 > m0 + 8.0f, up1 = mx1 > m1 + 8.0f;
                if (__any_sync(0xffffffffu, up0 || up1)) {
                    const float mn0 = up0 ? mx0 : m0, mn1 = up1 ? mx1 : m1;
                    const float al0 = ex2_fast(m0 - mn0), al1 = ex2_fast(m1 - mn1);
                    #pragma unroll
                    for (int k = 0; k < 8; k++) { o[k][0] *= al0; o[k][1] *= al1; o[k][2] *= al0; o[k][3] *= al1; }
                    l0 *= al0; l1 *= al1;
                    m0 = mn0; m1 = mn1;
                }
                float p[4];
                p[0] = ex2_fast(sc[0] - m0); p[1] = ex2_fast(sc[1] - m1);
                p[2] = ex2_fast(sc[2] - m0); p[3] = ex2_fast(sc[3] - m1);
                l0 += p[0] + p[2];
                l1 += p[1] + p[3];

                // ---- O^T += V^T P over this warp's 128 dims (rows not fetched: zero scale / values)
                if (KV_TYPE == QSA_TYPE_Q8_0) {
                    const uint32_t * V0 = reinterpret_cast<const uint32_t *>(Vt + (c0 + 0) * rb) + 34 * dh;
                    const uint32_t * V1 = reinterpret_cast<const uint32_t *>(Vt + (c0 + 1) * rb) + 34 * dh;
                    const uint32_t * V8 = reinterpret_cast<const uint32_t *>(Vt + (c0 + 8) * rb) + 34 * dh;
                    const uint32_t * V9 = reinterpret_cast<const uint32_t *>(Vt + (c0 + 9) * rb) + 34 * dh;
                    const uint16_t * VA = reinterpret_cast<const uint16_t *>(Vt + rA * rb) + 68 * dh;
                    const uint16_t * VB = reinterpret_cast<const uint16_t *>(Vt + rB * rb) + 68 * dh;
                    #pragma unroll
                    for (int gg = 0; gg < 4; gg++) {
                        float dA = f16_bits_to_f32(VA[17 * gg]);
                        float dB = f16_bits_to_f32(VB[17 * gg]);
                        dA = okA ? dA : 0.0f;
                        dB = okB ? dB : 0.0f;
                        uint32_t b[2];
                        b[0] = movmatrix_trans(pack_f16x2(p[0] * dA, p[1] * dA));
                        b[1] = movmatrix_trans(pack_f16x2(p[2] * dB, p[3] * dB));
                        uint32_t W0, W1, W2, W3;
                        if ((gg & 1) == 0) {
                            const int wi = 17 * (gg / 2) + r8;
                            W0 = __funnelshift_r(V0[wi], V0[wi + 1], 16);
                            W1 = __funnelshift_r(V1[wi], V1[wi + 1], 16);
                            W2 = __funnelshift_r(V8[wi], V8[wi + 1], 16);
                            W3 = __funnelshift_r(V9[wi], V9[wi + 1], 16);
                        } else {
                            const int wi = 17 * (gg / 2) + 9 + r8;
                            W0 = V0[wi]; W1 = V1[wi]; W2 = V8[wi]; W3 = V9[wi];
                        }
                        // V + 1152 (exact f16 integers); the bias is removed from both 16-dim
                        // tiles by -1152 x the column sums of the scaled P
                        const uint32_t am0[4] = {i8_pair_biased<0>(W0, W1), i8_pair_biased<1>(W0, W1),
                                                 i8_pair_biased<0>(W2, W3), i8_pair_biased<1>(W2, W3)};
                        const uint32_t am1[4] = {i8_pair_biased<2>(W0, W1), i8_pair_biased<3>(W0, W1),
                                                 i8_pair_biased<2>(W2, W3), i8_pair_biased<3>(W2, W3)};
                        mma_f16_16816(o[2 * gg], negb, b);
                        mma_f16_16816(o[2 * gg + 1], negb, b);
                        mma_f16_16816(o[2 * gg], am0, b);
                        mma_f16_16816(o[2 * gg + 1], am1, b);
                    }
                } else {
                    uint32_t b[2];
                    b[0] = movmatrix_trans(pack_f16x2(p[0], p[1]));
                    b[1] = movmatrix_trans(pack_f16x2(p[2], p[3]));
                    const uint32_t m01 = (((vm >> c0) & 1u) ? 0x0000ffffu : 0u) | (((vm >> (c0 + 1)) & 1u) ? 0xffff0000u : 0u);
                    const uint32_t m89 = (((vm >> (c0 + 8)) & 1u) ? 0x0000ffffu : 0u) | (((vm >> (c0 + 9)) & 1u) ? 0xffff0000u : 0u);
                    const int cl = 16 * cw + (lane & 7) + ((lane >> 4) << 3);   // ldmatrix row: cell
                    const int d8 = ((lane >> 3) & 1) << 3;                        // +8 dims for matrices 1, 3
                    #pragma unroll
                    for (int mm = 0; mm < 8; mm++) {
                        const int mt = 8 * dh + mm;
                        uint32_t a[4];
                        ldmatrix_x4_trans(a, Vt + cl * rb + 2 * (16 * mt + d8));
                        a[0] &= m01; a[1] &= m01; a[2] &= m89; a[3] &= m89;
                        mma_f16_16816(o[mm], a, b);
                    }
                }
            }
            // this warp is done with stage s: the producer may refill it
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty_bar[s]);
        }
    }
    __syncthreads();                                  // every warp past its last tile: stages are free

    // ---- merge the two 16-cell halves of each KV head (stage memory is free); the two dim-half
    // warps of a pair carry the same (m, l)
    #pragma unroll
    for (int off = 4; off < 32; off <<= 1) {
        l0 += __shfl_xor_sync(0xffffffffu, l0, off);
        l1 += __shfl_xor_sync(0xffffffffu, l1, off);
    }
    constexpr int HD2 = HEAD_DIM / 2;
    float * wm = reinterpret_cast<float *>(smem);               // [8 warps][8 heads] max
    float * wl = wm + ATT_CWARPS * 8;                            // [8][8] sum
    float * wf = wl + ATT_CWARPS * 8;                            // [8][8] merge factors
    float * cml = wf + ATT_CWARPS * 8;                           // [16] M, [16] L of the CTA
    float * wo = cml + 2 * HROWS;                                // [8][8][128] unnormalised O
    if (!producer) {
        if (r8 == 0) {
            wm[warp * 8 + 2 * j4] = m0; wm[warp * 8 + 2 * j4 + 1] = m1;
            wl[warp * 8 + 2 * j4] = l0; wl[warp * 8 + 2 * j4 + 1] = l1;
        }
        float * myo = wo + warp * 8 * HD2;
        if (KV_TYPE == QSA_TYPE_Q8_0) {
            #pragma unroll
            for (int gg = 0; gg < 4; gg++) {
                const int dim = 32 * gg + 4 * r8;
                *reinterpret_cast<float4 *>(myo + (2 * j4) * HD2 + dim) =
                    make_float4(o[2 * gg][0], o[2 * gg][2], o[2 * gg + 1][0], o[2 * gg + 1][2]);
                *reinterpret_cast<float4 *>(myo + (2 * j4 + 1) * HD2 + dim) =
                    make_float4(o[2 * gg][1], o[2 * gg][3], o[2 * gg + 1][1], o[2 * gg + 1][3]);
            }
        } else {
            #pragma unroll
            for (int mm = 0; mm < 8; mm++) {
                const int dim = 16 * mm + r8;
                myo[(2 * j4) * HD2 + dim]         = o[mm][0];
                myo[(2 * j4 + 1) * HD2 + dim]     = o[mm][1];
                myo[(2 * j4) * HD2 + dim + 8]     = o[mm][2];
                myo[(2 * j4 + 1) * HD2 + dim + 8] = o[mm][3];
            }
        }
    }
    __syncthreads();
    if (tid < HROWS) {   // row hr = 8*head + h: M over the head's two cell halves, L = sum l 2^(m - M)
        const int hh = tid >> 3, h = tid & 7;
        const int wa = 4 * hh, wb = 4 * hh + 2;                  // (head, cells 0-15 / 16-31, dims 0-127)
        const float M = fmaxf(wm[wa * 8 + h], wm[wb * 8 + h]);
        const float Mu = M == -INFINITY ? 0.0f : M;
        const float fa = exp2f(wm[wa * 8 + h] - Mu), fb = exp2f(wm[wb * 8 + h] - Mu);
        wf[wa * 8 + h] = fa; wf[wb * 8 + h] = fb;
        cml[tid] = M; cml[HROWS + tid] = wl[wa * 8 + h] * fa + wl[wb * 8 + h] * fb;
    }
    __syncthreads();
    // ---- the CTA's state: the final output (one chunk), or a partial for attn_merge_kernel
    const bool single = n_chunks == 1;
    float * po = part_o + ((size_t) t * max_chunks + chunk) * HROWS * HEAD_DIM;
    const int n_rows = d.n_head_kv * 8;
    for (int e4 = tid; e4 < HROWS * HEAD_DIM / 4; e4 += ATT_THREADS) {
        const int hr = (e4 * 4) / HEAD_DIM, hh = hr >> 3, h = hr & 7, d4 = e4 % (HEAD_DIM / 4);
        const int half = (d4 * 4) / HD2, dd4 = d4 % (HD2 / 4);
        const int wa = 4 * hh + half, wb = 4 * hh + 2 + half;    // the two cell halves, this dim half
        const float fa = wf[(4 * hh) * 8 + h], fb = wf[(4 * hh + 2) * 8 + h];
        const float4 va = reinterpret_cast<const float4 *>(wo + (wa * 8 + h) * HD2)[dd4];
        const float4 vb = reinterpret_cast<const float4 *>(wo + (wb * 8 + h) * HD2)[dd4];
        const float4 acc = make_float4(fa * va.x + fb * vb.x, fa * va.y + fb * vb.y,
                                       fa * va.z + fb * vb.z, fa * va.w + fb * vb.w);
        if (!single) {
            reinterpret_cast<float4 *>(po)[e4] = acc;
        } else if (stq) {
            state_put4(sdst, sq0 + 2 * HROWS + 4 * (size_t) e4, acc);
        } else if (hr < n_rows && h < d.gqa) {
            const float L = cml[HROWS + hr];
            const float inv = L > 0.0f ? 1.0f / L : 0.0f;
            out_store4(outs, outq + (size_t) hh * d.gqa * HEAD_DIM + (size_t) h * HEAD_DIM + 4 * d4,
                       make_float4(acc.x * inv, acc.y * inv, acc.z * inv, acc.w * inv));
        }
    }
    if (tid < 2 * HROWS) {
        if (!single) part_ml[((size_t) t * max_chunks + chunk) * 2 * HROWS + tid] = cml[tid];
        else if (stq) state_put(sdst, sq0 + tid, cml[tid]);
    }
}

// Merge of the per-CTA partials of the queries split over several chunks: CTA (t, row hr, 64-dim
// slice); out = sum_c 2^(m_c - M) O_c / sum_c 2^(m_c - M) l_c, M = max_c m_c (the state one CTA
// would have reached).  Thread = (float4 column of the slice, group of chunks), so that every
// thread has only a few independent partial loads in flight.  Launched programmatically behind
// attn_kernel.
constexpr int MERGE_COLS = 16;                        // float4 columns: 64 dims per CTA
constexpr int MERGE_GROUPS = MERGE_THREADS / MERGE_COLS;
// PRE: partial loads per thread issued up front (16 for long splits such as a batch-1 query over
// 134 chunks; 2 for batched decode, whose few chunks per query need few registers)
template <int PRE>
__global__ void __launch_bounds__(MERGE_THREADS) attn_merge_kernel(DevDesc d, const qsa_decode_item * __restrict__ items,
        int n_past0, const int * nsel_ws, int tiles_per_cta, int max_chunks,
        const float * part_o, const float * part_ml,
        OutSpec outs, StateDst sdst) {
    extern __shared__ float wsh[];                    // [max_chunks] weights
    __shared__ float red[2][MERGE_THREADS / 32];
    __shared__ float4 racc[MERGE_GROUPS][MERGE_COLS];
    const int t = blockIdx.x, hr = blockIdx.y;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int col = tid % MERGE_COLS, grp = tid / MERGE_COLS;
    const int d4 = blockIdx.z * MERGE_COLS + col;     // float4 index inside the row
    const int qpos = items ? items[t].n_past : n_past0 + t;
    const int g = hr >> 3, h = hr & 7;
    const bool live = g < d.n_head_kv && h < d.gqa;
    if (sdst.n == 0 && !live) return;
    pdl_wait();                                       // attn_kernel has completed: partials are written
    const bool pos_ok = qpos >= 0 && qpos < d.n_ctx;
    const int nsel = pos_ok ? max(0, min(ld_dep(nsel_ws + t), d.kb)) : 0;
    const int n_chunks = attn_n_chunks(d, nsel, tiles_per_cta);
    if (n_chunks <= 1) return;                        // written by the attention CTA itself
    // the partial rows do not depend on the weights: this thread's (up to PRE) loads go out
    // first, and the max / weight / sum rounds run while they are in flight
    const float4 * po = reinterpret_cast<const float4 *>(part_o + ((size_t) t * max_chunks * HROWS + hr) * HEAD_DIM) + d4;
    const size_t cstride = (size_t) HROWS * HEAD_DIM / 4;         // float4s between chunks
    float4 pre[PRE];
    #pragma unroll
    for (int k = 0; k < PRE; k++) {
        const int c = grp + k * MERGE_GROUPS;
        pre[k] = c < n_chunks ? ld_dep(po + (size_t) c * cstride) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
    const float * ml = part_ml + (size_t) t * max_chunks * 2 * HROWS;
    float M = -INFINITY;
    for (int c = tid; c < n_chunks; c += MERGE_THREADS) M = fmaxf(M, ld_dep(ml + c * 2 * HROWS + hr));
    M = warp_max(M);
    if (lane == 0) red[0][warp] = M;
    __syncthreads();
    M = red[0][0];
    #pragma unroll
    for (int w = 1; w < MERGE_THREADS / 32; w++) M = fmaxf(M, red[0][w]);
    const float Mu = M == -INFINITY ? 0.0f : M;
    float L = 0.0f;
    for (int c = tid; c < n_chunks; c += MERGE_THREADS) {
        const float w = exp2f(ld_dep(ml + c * 2 * HROWS + hr) - Mu);
        wsh[c] = w;
        L += ld_dep(ml + c * 2 * HROWS + HROWS + hr) * w;
    }
    #pragma unroll
    for (int o = 16; o > 0; o >>= 1) L += __shfl_xor_sync(0xffffffffu, L, o);
    if (lane == 0) red[1][warp] = L;
    __syncthreads();                                  // wsh and the partial sums are complete
    L = 0.0f;
    #pragma unroll
    for (int w = 0; w < MERGE_THREADS / 32; w++) L += red[1][w];
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    #pragma unroll
    for (int k = 0; k < PRE; k++) {
        const int c = grp + k * MERGE_GROUPS;
        const float w = c < n_chunks ? wsh[c] : 0.0f;
        acc.x += w * pre[k].x; acc.y += w * pre[k].y; acc.z += w * pre[k].z; acc.w += w * pre[k].w;
    }
    #pragma unroll 4
    for (int c = grp + PRE * MERGE_GROUPS; c < n_chunks; c += MERGE_GROUPS) {   // longer splits
        const float4 v = ld_dep(po + (size_t) c * cstride);
        const float w = wsh[c];
        acc.x += w * v.x; acc.y += w * v.y; acc.z += w * v.z; acc.w += w * v.w;
    }
    racc[grp][col] = acc;
    __syncthreads();
    if (tid < MERGE_COLS) {
        float4 s = racc[0][tid];
        #pragma unroll
        for (int k = 1; k < MERGE_GROUPS; k++) {
            const float4 v = racc[k][tid];
            s.x += v.x; s.y += v.y; s.z += v.z; s.w += v.w;
        }
        if (sdst.n > 0) {
            const size_t sq0 = (size_t) t * (2 * HROWS + HROWS * HEAD_DIM);
            state_put4(sdst, sq0 + 2 * HROWS + (size_t) hr * HEAD_DIM + 4 * d4, s);
            if (blockIdx.z == 0 && tid == 0) { state_put(sdst, sq0 + hr, M); state_put(sdst, sq0 + HROWS + hr, L); }
        } else {
            const float inv = L > 0.0f ? 1.0f / L : 0.0f;
            out_store4(outs, ((size_t) t * d.n_head + g * d.gqa + h) * HEAD_DIM + 4 * d4,
                       make_float4(s.x * inv, s.y * inv, s.z * inv, s.w * inv));
        }
    }
}

// The merge for queries split over at most MERGE_SMALL_CHUNKS chunks (batched decode, short
// prefill chunks): CTA = query, thread = (row hr, float4 column); every thread loads its row's
// (m, l) and its column of every partial at once and forms the same M, weights and L as
// attn_merge_kernel.  Launched programmatically behind attn_kernel.
constexpr int MERGE_SMALL_CHUNKS = 8;
constexpr int MERGE_SMALL_THREADS = HROWS * HEAD_DIM / 4;

__global__ void __launch_bounds__(MERGE_SMALL_THREADS) attn_merge_small_kernel(DevDesc d,
        const qsa_decode_item * __restrict__ items, int n_past0, const int * nsel_ws, int tiles_per_cta, int max_chunks,
        const float * part_o, const float * part_ml, OutSpec outs, StateDst sdst) {
    const int t = blockIdx.x, tid = threadIdx.x;
    const int hr = tid / (HEAD_DIM / 4), d4 = tid % (HEAD_DIM / 4);
    const int g = hr >> 3, h = hr & 7;
    const int qpos = items ? items[t].n_past : n_past0 + t;
    const bool live = g < d.n_head_kv && h < d.gqa;
    if (sdst.n == 0 && !live) return;
    pdl_wait();                                       // attn_kernel has completed: partials are written
    const bool pos_ok = qpos >= 0 && qpos < d.n_ctx;
    const int nsel = pos_ok ? max(0, min(ld_dep(nsel_ws + t), d.kb)) : 0;
    const int n_chunks = min(attn_n_chunks(d, nsel, tiles_per_cta), MERGE_SMALL_CHUNKS);
    if (n_chunks <= 1) return;                        // written by the attention CTA itself
    const float * ml = part_ml + (size_t) t * max_chunks * 2 * HROWS;
    const float4 * po = reinterpret_cast<const float4 *>(part_o + ((size_t) t * max_chunks * HROWS + hr) * HEAD_DIM) + d4;
    const size_t cstride = (size_t) HROWS * HEAD_DIM / 4;         // float4s between chunks
    float mc[MERGE_SMALL_CHUNKS], lc[MERGE_SMALL_CHUNKS];
    float4 oc[MERGE_SMALL_CHUNKS];
    #pragma unroll
    for (int c = 0; c < MERGE_SMALL_CHUNKS; c++) {
        if (c < n_chunks) {
            mc[c] = ld_dep(ml + c * 2 * HROWS + hr);
            lc[c] = ld_dep(ml + c * 2 * HROWS + HROWS + hr);
            oc[c] = ld_dep(po + (size_t) c * cstride);
        } else {
            mc[c] = -INFINITY; lc[c] = 0.0f; oc[c] = make_float4(0.f, 0.f, 0.f, 0.f);
        }
    }
    float M = -INFINITY;
    #pragma unroll
    for (int c = 0; c < MERGE_SMALL_CHUNKS; c++) M = fmaxf(M, mc[c]);
    const float Mu = M == -INFINITY ? 0.0f : M;
    float L = 0.0f;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    #pragma unroll
    for (int c = 0; c < MERGE_SMALL_CHUNKS; c++) {
        if (c >= n_chunks) break;
        const float w = exp2f(mc[c] - Mu);
        L += lc[c] * w;
        acc.x += w * oc[c].x; acc.y += w * oc[c].y; acc.z += w * oc[c].z; acc.w += w * oc[c].w;
    }
    if (sdst.n > 0) {
        const size_t sq0 = (size_t) t * (2 * HROWS + HROWS * HEAD_DIM);
        state_put4(sdst, sq0 + 2 * HROWS + (size_t) hr * HEAD_DIM + 4 * d4, acc);
        if (d4 == 0) { state_put(sdst, sq0 + hr, M); state_put(sdst, sq0 + HROWS + hr, L); }
    } else {
        const float inv = L > 0.0f ? 1.0f / L : 0.0f;
        out_store4(outs, ((size_t) t * d.n_head + g * d.gqa + h) * HEAD_DIM + 4 * d4,
                   make_float4(acc.x * inv, acc.y * inv, acc.z * inv, acc.w * inv));
    }
}

template <int KV_TYPE, int NKV>
cudaError_t attn_set_attr_one() {
    return cudaFuncSetAttribute(attn_kernel<KV_TYPE, NKV>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                attn_smem_bytes<KV_TYPE>(MAX_KB));
}

cudaError_t attn_set_attrs() {
    cudaError_t e = attn_set_attr_one<QSA_TYPE_Q8_0, 2>();
    if (e == cudaSuccess) e = attn_set_attr_one<QSA_TYPE_Q8_0, 1>();
    if (e == cudaSuccess) e = attn_set_attr_one<QSA_TYPE_F16, 2>();
    if (e == cudaSuccess) e = attn_set_attr_one<QSA_TYPE_F16, 1>();
    return e;
}

int attn_tile_cells() { return ATT_CELLS; }

int attn_state_rows() { return HROWS; }

int attn_resident_ctas(int type_k) {
    return 148 * (type_k == QSA_TYPE_Q8_0 ? AttnCfg<QSA_TYPE_Q8_0>::MIN_CTAS : AttnCfg<QSA_TYPE_F16>::MIN_CTAS);
}

cudaError_t launch_attn(const DevDesc & d, cudaStream_t st, bool chained, int n_q, const qsa_decode_item * items,
        qsa_layer_cache cache0, int n_past0, const void * q, int q_type, const int * sel_ws, const int * nsel_ws,
        int tiles_per_cta, int max_chunks, float * part_o, float * part_ml, OutSpec outs, uint32_t * status,
        const StateDst & sdst) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned) max_chunks, (unsigned) n_q);
    cfg.blockDim = dim3(ATT_THREADS);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;   // prologue overlaps the select
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = chained ? 1 : 0;     // the first kernel of a call waits for all earlier work
    cudaError_t e;
    cfg.dynamicSmemBytes = d.type_k == QSA_TYPE_Q8_0 ? attn_smem_bytes<QSA_TYPE_Q8_0>(d.kb) : attn_smem_bytes<QSA_TYPE_F16>(d.kb);
    // A grid of at most one CTA per SM asks for the most shared memory the kernel allows, so that no
    // SM takes two of its CTAs: launched behind the selection, whose CTAs hold most SMs, two q8_0
    // CTAs would otherwise pair up on the SMs that come free first.
    if ((int64_t) max_chunks * n_q <= 148 && d.type_k == QSA_TYPE_Q8_0)
        cfg.dynamicSmemBytes = attn_smem_bytes<QSA_TYPE_Q8_0>(MAX_KB);
#define QSA_LAUNCH_ATTN(T, N) cudaLaunchKernelEx(&cfg, attn_kernel<T, N>, d, items, cache0, n_past0, q, q_type, sel_ws, \
                                                 nsel_ws, tiles_per_cta, max_chunks, part_o, part_ml, outs, status, sdst)
    if (d.type_k == QSA_TYPE_Q8_0) e = d.n_head_kv == 2 ? QSA_LAUNCH_ATTN(QSA_TYPE_Q8_0, 2) : QSA_LAUNCH_ATTN(QSA_TYPE_Q8_0, 1);
    else                           e = d.n_head_kv == 2 ? QSA_LAUNCH_ATTN(QSA_TYPE_F16, 2) : QSA_LAUNCH_ATTN(QSA_TYPE_F16, 1);
#undef QSA_LAUNCH_ATTN
    if (e != cudaSuccess || max_chunks <= 1) return e;
    cudaLaunchConfig_t mc = cfg;
    mc.numAttrs = 1;                    // the merge follows the attention of this call
    if (max_chunks <= MERGE_SMALL_CHUNKS) {
        mc.gridDim = dim3((unsigned) n_q);
        mc.blockDim = dim3(MERGE_SMALL_THREADS);
        mc.dynamicSmemBytes = 0;
        return cudaLaunchKernelEx(&mc, attn_merge_small_kernel, d, items, n_past0, nsel_ws, tiles_per_cta, max_chunks,
                                  (const float *) part_o, (const float *) part_ml, outs, sdst);
    }
    mc.gridDim = dim3((unsigned) n_q, HROWS, HEAD_DIM / (4 * MERGE_COLS));
    mc.blockDim = dim3(MERGE_THREADS);
    mc.dynamicSmemBytes = (size_t) max_chunks * 4;
    if (max_chunks > 2 * MERGE_GROUPS)
        return cudaLaunchKernelEx(&mc, attn_merge_kernel<16>, d, items, n_past0, nsel_ws, tiles_per_cta, max_chunks,
                                  (const float *) part_o, (const float *) part_ml, outs, sdst);
    return cudaLaunchKernelEx(&mc, attn_merge_kernel<2>, d, items, n_past0, nsel_ws, tiles_per_cta, max_chunks,
                              (const float *) part_o, (const float *) part_ml, outs, sdst);
}

}  // namespace qsa
