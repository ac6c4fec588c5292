// qsa_select.cu -- lightning-indexer scores and top-k block selection.
//
// Reference: decode scores src/qwfn_graph.cpp:478-492, prefill :277-293 (mul_mat of the F16
// pooled keys with the indexer query converted to F16, relu per head, sum over heads, + bias);
// ggml_top_k + block->cell expansion :493-495 / :295-306; the bias rules of
// src/qwfn_engine.cpp:748-753 (decode) and :936-950 (prefill), applied here as a rule:
//   visible  = blocks whole at the query, (b+1)*r <= q+1           (bias 0)
//   forced   = window > 0: blocks b_q-nf+1..b_q; window == 0: b_q while incomplete (bias +1e9)
//   selected = forced + the (KB - |forced|) best visible non-forced blocks; ties -> lower index.
//
// One kernel: CTAs of a query score disjoint block ranges into the workspace; the last CTA of
// the query to finish (atomic arrival counter, no waiting) selects on a few of its warps with an
// exact radix select over the scores and writes the ascending block list.
#include "qsa_kernels.cuh"

namespace qsa {

constexpr int SEL_THREADS = SEL_THREADS_HOST;

// Score blocks [b_begin, b_end) of one query: 16 lanes per block row (8 dims = 16 bytes each), a
// warp on SCORE_U row pairs at a time (their loads in flight together).  Products of two f16
// values are exact in f32; they are summed in double (exact for these magnitudes) and rounded
// once, so the result does not depend on the summation order.
constexpr int SCORE_U = 8;

// This warp's rows of the batch at b0 (rows b0 + u*step + half); pooled keys the append before
// this grid may have written, read after its pdl_wait.
__device__ __forceinline__ void score_load(const uint16_t * pool, int b0, int b_end, int step, uint4 (&w)[SCORE_U]) {
    const int half = (threadIdx.x >> 4) & 1, sub = threadIdx.x & 15;
    #pragma unroll
    for (int u = 0; u < SCORE_U; u++) {
        const int b = b0 + u * step + half;
        w[u] = b < b_end ? ld_dep(reinterpret_cast<const uint4 *>(pool + (size_t) b * MAX_IDX_DIM + 8 * sub))
                         : make_uint4(0, 0, 0, 0);
    }
}

__device__ __forceinline__ void score_range(const DevDesc & d, const uint16_t * pool,
        const float (&qf)[4][8], int b_begin, int b_end, float * __restrict__ scores, const uint4 (&first)[SCORE_U]) {
    const int warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    const int half = (threadIdx.x >> 4) & 1, sub = threadIdx.x & 15;
    const int step = 2 * nw;
    uint4 w[SCORE_U];
    #pragma unroll
    for (int u = 0; u < SCORE_U; u++) w[u] = first[u];      // the first batch was loaded by the caller
    #pragma unroll 1
    for (int b0 = b_begin + 2 * warp; b0 < b_end; b0 += SCORE_U * step) {
        if (b0 != b_begin + 2 * warp) score_load(pool, b0, b_end, step, w);
        #pragma unroll
        for (int u = 0; u < SCORE_U; u++) {
            if (b0 + u * step >= b_end) break;           // this warp's remaining rows are past the range
            const int b = b0 + u * step + half;
            const uint32_t ws[4] = {w[u].x, w[u].y, w[u].z, w[u].w};
            float pk[8];
            #pragma unroll
            for (int i = 0; i < 4; i++) {
                pk[2 * i]     = f16_bits_to_f32((uint16_t) (ws[i] & 0xffff));
                pk[2 * i + 1] = f16_bits_to_f32((uint16_t) (ws[i] >> 16));
            }
            double hs = 0.0;
            #pragma unroll
            for (int h = 0; h < 4; h++) {
                if (h >= d.idx_n_head) break;
                double acc = 0.0;
                #pragma unroll
                for (int e = 0; e < 8; e++) acc += (double) __fmul_rn(pk[e], qf[h][e]);
                acc = warp_sum16_d(acc);
                const float dot = (float) acc;
                hs += (double) (dot > 0.0f ? dot : 0.0f);
            }
            if (b < b_end && sub == 0) scores[b] = (float) hs;
        }
    }
}

// Forced block range of the query at q: [f_lo, f_hi] (empty when f_lo > f_hi).
__device__ __forceinline__ void forced_range(const DevDesc & d, int q, int & f_lo, int & f_hi) {
    const int bq = q / d.ratio;
    if (d.window > 0) { f_lo = max(0, bq - d.n_force + 1); f_hi = bq; }
    else if ((q + 1) % d.ratio != 0) { f_lo = bq; f_hi = bq; }
    else { f_lo = 1; f_hi = 0; }
}

constexpr int SEL_BINS = 256;      // one radix digit: 8 bits
constexpr int LIST_MAX = 4096;     // entries of a cut bin collected for the later digits
constexpr int RANK_MAX = 32;       // a cut bin this small is ranked directly

// Selection scratch of the last CTA of a query.  The digit histograms are triple-buffered: a
// level's pass clears the buffer of the level after next while slower warps may still search the
// previous one.
struct SelSmem {
    alignas(16) unsigned hist[3][SEL_BINS];
    unsigned long long stage[RANK_MAX];   // the entries of a small cut bin
    int list[LIST_MAX];
    int slist[MAX_KB];                    // the selected blocks, ascending
    int wcount[SEL_THREADS_HOST / 32];
    int nlist, nstage;
};

// Threads of the selection (the first warps of the CTA) meet at named barrier 1.
__device__ __forceinline__ void sel_sync(int n_threads) {
    asm volatile("bar.sync 1, %0;" :: "r"(n_threads) : "memory");
}

struct Cut { int bin, remaining, in_bin; };

// The bin of histogram h holding the `remaining`-th entry counted from the top bin down, how many
// of its entries are still to take, and how many it holds.  Every warp computes it (no barrier).
__device__ Cut find_cut(const unsigned * h, int remaining) {
    const int lane = threadIdx.x & 31;
    const uint4 a = *reinterpret_cast<const uint4 *>(h + 248 - 8 * lane);
    const uint4 b = *reinterpret_cast<const uint4 *>(h + 252 - 8 * lane);
    const unsigned c[8] = {b.w, b.z, b.y, b.x, a.w, a.z, a.y, a.x};     // bins 255-8l down to 248-8l
    int own = 0;
    #pragma unroll
    for (int k = 0; k < 8; k++) own += (int) c[k];
    int incl = own;
    #pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int v = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += v;
    }
    const int above = incl - own;
    const bool hit = above < remaining && incl >= remaining;
    const unsigned m = __ballot_sync(0xffffffffu, hit);
    Cut r{0, 0, 0};
    if (hit) {
        int cum = above;
        #pragma unroll
        for (int k = 0; k < 8; k++) {
            if (cum + (int) c[k] >= remaining) { r.bin = 255 - 8 * lane - k; r.remaining = remaining - cum; r.in_bin = (int) c[k]; break; }
            cum += (int) c[k];
        }
    }
    const int src = m ? __ffs(m) - 1 : 0;
    r.bin = __shfl_sync(0xffffffffu, r.bin, src);
    r.remaining = __shfl_sync(0xffffffffu, r.remaining, src);
    r.in_bin = __shfl_sync(0xffffffffu, r.in_bin, src);
    return r;
}

// Selection of one query by the first nws warps of the last CTA.
//
// Candidates are the blocks [lo_c, c_end); the forced blocks f_lo.. (all above c_end) are added
// unless sharded.  The rule "highest score, ties to the lower block" is the order of the 63-bit
// composite (score bits << 32) | (c_end - 1 - b): the want-th largest composite K is found by an
// exact radix select over 8-bit digits (the first, the score's exponent, counted while the scores
// are loaded; a list of the cut bin's entries replaces the full range once it holds at most
// LIST_MAX; a cut bin of at most RANK_MAX is ranked directly), and the blocks with composite >= K
// are written in ascending order by a ballot compaction.  The loops are kept rolled: this code
// runs once per query, usually with its instructions not in any cache.
//
// Sharded mode (cand_scores != null): forced blocks are left to the global merge and each kept
// block's score is written beside it.  Replicated indexer caches (shard_ri): sel_out holds the
// global list and the attention's list the run of it inside [shard_blk0, shard_blk1).
__device__ void select_blocks(const DevDesc & d, const float * sc_g, float * ssc, unsigned * balls, SelSmem & sm,
                              int lo_c, int c_end, int f_lo, int n_forced, int nws,
                              int * __restrict__ sel, int * __restrict__ nsel_out, int * __restrict__ sel_out,
                              float * __restrict__ cand_scores) {
    const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5, ns = 32 * nws;
    const bool shard = cand_scores != nullptr;
    const int n_c = c_end - lo_c;
    const int want = max(0, d.kb - n_forced);
    auto comp = [&](int b) -> unsigned long long {
        return ((unsigned long long) __float_as_uint(ssc[b]) << 32) | (unsigned) (c_end - 1 - b);
    };
    // 1. the candidates' scores into shared memory (16-byte loads, four in flight per thread: score
    //    rows are 16-byte aligned; written by the other CTAs of this grid, read after the arrival's
    //    acquire), with the histogram of the first digit (score bits 30..23), counted from shared
    //    memory by a short loop.  Zero scores (every head cut by the relu, about half of the keys)
    //    are counted per warp.
    {
        constexpr int U = 4;
        const int i0 = lo_c >> 2, i1 = (c_end + 3) >> 2;
        #pragma unroll 1
        for (int base = i0; base < i1; base += U * ns) {
            float4 v[U];
            #pragma unroll
            for (int u = 0; u < U; u++) {
                const int i = base + u * ns + tid;
                v[u] = i < i1 ? __ldcg(reinterpret_cast<const float4 *>(sc_g) + i) : make_float4(0.f, 0.f, 0.f, 0.f);
            }
            #pragma unroll
            for (int u = 0; u < U; u++) {
                const int i = base + u * ns + tid;
                if (i < i1) reinterpret_cast<float4 *>(ssc)[i] = v[u];
            }
            int n_zero = 0;
            #pragma unroll 1
            for (int u = 0; u < U; u++) {
                const int i = base + u * ns + tid;
                if (i >= i1) break;
                const float4 x = reinterpret_cast<const float4 *>(ssc)[i];
                const float e[4] = {x.x, x.y, x.z, x.w};
                #pragma unroll
                for (int k = 0; k < 4; k++) {
                    const int b = 4 * i + k;
                    const unsigned key = __float_as_uint(e[k]);
                    if (b < lo_c || b >= c_end) continue;
                    if (key) atomicAdd(&sm.hist[0][(key >> 23) & 0xffu], 1u);
                    else n_zero++;
                }
            }
            #pragma unroll
            for (int o = 16; o > 0; o >>= 1) n_zero += __shfl_xor_sync(0xffffffffu, n_zero, o);
            if (lane == 0 && n_zero) atomicAdd(&sm.hist[0][0], (unsigned) n_zero);
        }
    }
    sel_sync(ns);
    // 2. the threshold composite K: take block b iff comp(b) >= K
    unsigned long long K = 0ull;                      // fewer candidates than wanted: all
    if (want == 0) K = ~0ull;                         // none (composites are below 2^63)
    else if (n_c > want) {
        int remaining = want;
        unsigned long long prefix = 0ull, pmask = 1ull << 63;
        int shift = 55, width = 8;
        bool from_list = false;
        int nlist = 0;
        #pragma unroll 1
        for (int level = 0; level < 9; level++) {
            const Cut c = find_cut(sm.hist[level % 3], remaining);
            prefix |= (unsigned long long) c.bin << shift;
            pmask |= (unsigned long long) ((1u << width) - 1u) << shift;
            remaining = c.remaining;
            if (c.in_bin == remaining || shift == 0) { K = prefix; break; }
            const bool rank = c.in_bin <= RANK_MAX;
            // a pass over the source (the full range, or the list): either the bin's entries to
            // the stage (a small bin), or the next digit's histogram (collecting the bin's
            // entries on the way once the bin is small enough for the list)
            const bool collect = !rank && !from_list && c.in_bin <= LIST_MAX;
            int dshift = 0;
            unsigned dmask = 0u;
            unsigned * hcur = sm.hist[(level + 1) % 3];
            if (!rank) {
                const int hb = shift - 1;
                width = min(8, hb + 1);
                dshift = hb + 1 - width;
                dmask = (1u << width) - 1u;
                unsigned * hnext = sm.hist[(level + 2) % 3];
                for (int i = tid; i < SEL_BINS; i += ns) hnext[i] = 0u;
            }
            const int n = from_list ? nlist : n_c;
            // over many candidates the keys of four iterations are read ahead (this loop then runs
            // long enough for its wider code to pay); short passes keep the compact loop
            const int p_fast = (!from_list && n > 4096) ? n - n % (4 * ns) : 0;
            #pragma unroll 1
            for (int p0 = tid; p0 < p_fast; p0 += 4 * ns) {
                unsigned long long Cs[4];
                #pragma unroll
                for (int u = 0; u < 4; u++) Cs[u] = comp(lo_c + p0 + u * ns);
                #pragma unroll
                for (int u = 0; u < 4; u++) {
                    const unsigned long long C = Cs[u];
                    if ((C & pmask) != prefix) continue;
                    if (rank) {
                        const int slot = atomicAdd(&sm.nstage, 1);
                        if (slot < RANK_MAX) sm.stage[slot] = C;
                        continue;
                    }
                    if (collect) {
                        const int slot = atomicAdd(&sm.nlist, 1);
                        if (slot < LIST_MAX) sm.list[slot] = lo_c + p0 + u * ns;
                    }
                    atomicAdd(hcur + ((unsigned) (C >> dshift) & dmask), 1u);
                }
            }
            #pragma unroll 1
            for (int p = p_fast + tid; p < n; p += ns) {
                const int b = from_list ? sm.list[p] : lo_c + p;
                const unsigned long long C = comp(b);
                if ((C & pmask) != prefix) continue;
                if (rank) {
                    const int slot = atomicAdd(&sm.nstage, 1);
                    if (slot < RANK_MAX) sm.stage[slot] = C;
                    continue;
                }
                if (collect) {
                    const int slot = atomicAdd(&sm.nlist, 1);
                    if (slot < LIST_MAX) sm.list[slot] = b;
                }
                atomicAdd(hcur + ((unsigned) (C >> dshift) & dmask), 1u);
            }
            sel_sync(ns);
            if (rank) {                               // every warp ranks the staged entries
                const int cnt = min(sm.nstage, RANK_MAX);
                const unsigned long long mine = lane < cnt ? sm.stage[lane] : 0ull;
                int r = 0;
                #pragma unroll 1
                for (int j = 0; j < cnt; j++) r += sm.stage[j] > mine;
                const unsigned hit = __ballot_sync(0xffffffffu, lane < cnt && r == remaining - 1);
                const int src = hit ? __ffs(hit) - 1 : 0;
                K = ((unsigned long long) __shfl_sync(0xffffffffu, (unsigned) (mine >> 32), src) << 32) |
                    __shfl_sync(0xffffffffu, (unsigned) mine, src);
                break;
            }
            shift = dshift;
            if (collect) { from_list = true; nlist = min(sm.nlist, LIST_MAX); }
        }
    }
    // 3. ordered compaction: warp w covers a contiguous run of R rounds of 32 candidates
    const int R = (n_c + ns - 1) / ns;
    const int start = lo_c + w * R * 32, end = min(c_end, start + R * 32);
    int cnt = 0;
    const int r_fast = R >= 8 ? R - R % 4 : 0;        // many rounds: four in flight
    #pragma unroll 1
    for (int r0 = 0; r0 < r_fast; r0 += 4) {
        bool tk[4];
        #pragma unroll
        for (int u = 0; u < 4; u++) {
            const int b = start + 32 * (r0 + u) + lane;
            tk[u] = b < end && comp(b) >= K;
        }
        #pragma unroll
        for (int u = 0; u < 4; u++) {
            const unsigned m = __ballot_sync(0xffffffffu, tk[u]);
            if (lane == 0) balls[w * R + r0 + u] = m;
            cnt += __popc(m);
        }
    }
    #pragma unroll 1
    for (int r = r_fast; r < R; r++) {
        const int b = start + 32 * r + lane;
        const unsigned m = __ballot_sync(0xffffffffu, b < end && comp(b) >= K);
        if (lane == 0) balls[w * R + r] = m;
        cnt += __popc(m);
    }
    if (lane == 0) sm.wcount[w] = cnt;
    sel_sync(ns);
    int base = 0, total = 0;
    #pragma unroll 1
    for (int v = 0; v < nws; v++) {
        const int x = sm.wcount[v];
        base += v < w ? x : 0;
        total += x;
    }
    #pragma unroll 1
    for (int r = 0; r < R; r++) {
        const unsigned m = balls[w * R + r];
        const int pos = base + __popc(m & ((1u << lane) - 1u));
        if (((m >> lane) & 1u) && pos < d.kb) sm.slist[pos] = start + 32 * r + lane;
        base += __popc(m);
    }
    int n = min(total, d.kb);
    if (!shard) {
        for (int i = tid; i < n_forced; i += ns)
            if (total + i < d.kb) sm.slist[total + i] = f_lo + i;
        n = min(total + n_forced, d.kb);
    }
    sel_sync(ns);
    // 4. the lists, coalesced
    int a0 = 0, m_att = n;                            // the attention's run of the list
    if (d.shard_ri) {
        auto lower = [&](int x) {
            int lo = 0, hi = n;
            while (lo < hi) { const int mid = (lo + hi) >> 1; if (sm.slist[mid] < x) lo = mid + 1; else hi = mid; }
            return lo;
        };
        a0 = lower(d.shard_blk0);
        m_att = lower(d.shard_blk1) - a0;
    }
    for (int i = tid; i < d.kb; i += ns) {
        const int b = i < n ? sm.slist[i] : -1;
        if (sel_out) sel_out[i] = b;
        if (d.shard_ri) sel[i] = i < m_att ? sm.slist[a0 + i] : -1;
        else if (i < n) sel[i] = b;
        else if (shard) sel[i] = -1;
        if (shard) cand_scores[i] = i < n ? ssc[b] : 0.0f;
    }
    if (tid == 0) *nsel_out = d.shard_ri ? m_att : n;
}

// grid = (score CTAs per query, n_queries).  Query t: position q_pos(t), pooled cache `pool`.
// Decode: items != null (per-query caches and n_past); prefill: one cache, q = n_past0 + t.
__global__ void __launch_bounds__(SEL_THREADS, 1) score_select_kernel(DevDesc d,
        const qsa_decode_item * __restrict__ items, const uint16_t * __restrict__ pool0, int n_past0,
        const float * __restrict__ q_idx, int blocks_per_cta,
        float * __restrict__ scores_ws, int scores_stride, unsigned * __restrict__ counters,
        int * __restrict__ sel_ws, int * __restrict__ nsel_ws, int * __restrict__ sel_out,
        uint32_t * __restrict__ status, float * __restrict__ cand_scores) {
    extern __shared__ __align__(16) unsigned char dyn_smem[];
    __shared__ SelSmem sm;
    __shared__ bool is_last;
    pdl_trigger();
    if (threadIdx.x < 2 * SEL_BINS) (&sm.hist[0][0])[threadIdx.x] = 0u;     // the first two digits' bins
    if (threadIdx.x == 0) { sm.nlist = 0; sm.nstage = 0; }
    const int t = blockIdx.y;
    const int q = items ? items[t].n_past : n_past0 + t;
    const uint16_t * pool = items ? items[t].cache.pool : pool0;
    // the blocks that compete: all ([0, INT_MAX)) unless the indexer caches are sharded too
    const int blo = d.shard_ri ? 0 : d.shard_blk0, bhi = d.shard_ri ? INT_MAX : d.shard_blk1;
    if (blo != 0) pool = shard_row(pool, (int64_t) blo, 0, (int64_t) d.idx_dim * 2);   // address of block 0
    const bool bad = q < 0 || q >= d.n_ctx || (q + 1) / d.ratio > scores_stride;
    if (bad && threadIdx.x == 0 && blockIdx.x == 0) set_status(status, DEV_BAD_POS);
    const int n_vis = bad ? 0 : (q + 1) / d.ratio;
    float * sc = scores_ws + (size_t) t * scores_stride;
    // candidates only: the forced blocks are the top of the visible range and never compete
    int f_lo = 1, f_hi = 0;
    if (!bad) forced_range(d, q, f_lo, f_hi);
    const int n_forced = f_hi >= f_lo ? f_hi - f_lo + 1 : 0;
    const int cand_hi = n_forced ? min(n_vis, f_lo) : n_vis;

    // Decode with a window: this step's append writes only the query's own block (its pooled
    // key included), which is forced, so scoring need not wait for it; the wait moves to the exit
    // (the attention, launched behind this grid, still finds the appended row).
    const bool defer_wait = items != nullptr && d.window > 0;
    if (!bad) {
        const int b0 = blo + blockIdx.x * blocks_per_cta;
        const int b1 = min(min(cand_hi, bhi), b0 + blocks_per_cta);
        if (!defer_wait) pdl_wait();             // the append of this step (pooled keys) is complete
        // this warp's first batch of rows is requested before the query is read: the loads overlap
        const int sub = threadIdx.x & 15;
        uint4 first[SCORE_U];
        score_load(pool, b0 + 2 * (int) (threadIdx.x >> 5), b1, 2 * (int) (blockDim.x >> 5), first);
        float qf[4][8];
        #pragma unroll
        for (int h = 0; h < 4; h++)
            #pragma unroll
            for (int e = 0; e < 8; e++)
                qf[h][e] = h < d.idx_n_head
                    ? f16_bits_to_f32(f32_to_f16_bits(q_idx[((size_t) t * d.idx_n_head + h) * d.idx_dim + 8 * sub + e]))
                    : 0.0f;
        if (b0 < b1) score_range(d, pool, qf, b0, b1, sc, first);
    }
    if (bad && !defer_wait) pdl_wait();
    // Arrival: the last CTA of this query selects.  The barrier orders the CTA's score stores
    // before thread 0's release; its acquire orders the other CTAs' stores before our reads.
    __syncthreads();
    if (threadIdx.x == 0) {
        unsigned prev;
        asm volatile("atom.add.acq_rel.gpu.u32 %0, [%1], 1;" : "=r"(prev) : "l"(counters + t) : "memory");
        is_last = prev == gridDim.x - 1;
        if (is_last) counters[t] = 0;          // leave the counter at zero for the next call
    }
    __syncthreads();
    // the selection runs on up to 16 warps (one per 128 candidates); the others leave
    const int lo_c = max(blo, 0), hi_c = min(bhi, n_vis);
    const int c_end = max(lo_c, n_forced ? min(hi_c, f_lo) : hi_c);       // candidates [lo_c, c_end)
    const int nws = min(SEL_THREADS / 32, max(1, (c_end - lo_c + 127) / 128));
    if (!is_last || (int) threadIdx.x >= 32 * nws) {
        if (defer_wait) pdl_wait();
        return;
    }
    if (bad) {
        for (int i = threadIdx.x; i < d.kb; i += 32 * nws) {
            sel_ws[(size_t) t * d.kb + i] = -1;
            if (sel_out) sel_out[(size_t) t * d.kb + i] = -1;
            if (cand_scores) cand_scores[(size_t) t * d.kb + i] = 0.0f;
        }
        if (threadIdx.x == 0) nsel_ws[t] = 0;
    } else {
        float * ssc = reinterpret_cast<float *>(dyn_smem);
        unsigned * balls = reinterpret_cast<unsigned *>(dyn_smem + (size_t) scores_stride * 4);
        select_blocks(d, sc, ssc, balls, sm, lo_c, c_end, f_lo, n_forced, nws, sel_ws + (size_t) t * d.kb, nsel_ws + t,
                      sel_out ? sel_out + (size_t) t * d.kb : nullptr,
                      cand_scores ? cand_scores + (size_t) t * d.kb : nullptr);
    }
    if (defer_wait) pdl_wait();                  // the append is complete before this grid is
}

}  // namespace qsa
