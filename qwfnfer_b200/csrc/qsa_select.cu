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
// the query to finish (atomic arrival counter, no waiting) selects with a radix select over the
// scores and writes the ascending block list.
#include <cub/block/block_scan.cuh>

#include "qsa_kernels.cuh"

namespace qsa {

constexpr int SEL_THREADS = SEL_THREADS_HOST;
static_assert(MAX_KB <= SEL_THREADS, "one kept block per selection thread");

// Score blocks [b_begin, b_end) of one query: 16 lanes per block row (8 dims = 16 bytes each).
// Products of two f16 values are exact in f32; they are summed in double (exact for these
// magnitudes) and rounded once, so the result does not depend on the summation order.
__device__ __forceinline__ void score_range(const DevDesc & d, const uint16_t * pool,
        const float (&qf)[4][8], int b_begin, int b_end, float * __restrict__ scores) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    const int half = lane >> 4, sub = lane & 15;
    for (int b0 = b_begin + 2 * warp; b0 < b_end; b0 += 2 * nw) {
        const int b = b0 + half;
        const bool ok = b < b_end;
        uint4 w = make_uint4(0, 0, 0, 0);
        // pooled keys the append before this grid may have written (read after its pdl_wait)
        if (ok) w = ld_dep(reinterpret_cast<const uint4 *>(pool + (size_t) b * MAX_IDX_DIM + 8 * sub));
        const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
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
        if (ok && sub == 0) scores[b] = (float) hs;
    }
}

// Forced block range of the query at q: [f_lo, f_hi] (empty when f_lo > f_hi).
__device__ __forceinline__ void forced_range(const DevDesc & d, int q, int & f_lo, int & f_hi) {
    const int bq = q / d.ratio;
    if (d.window > 0) { f_lo = max(0, bq - d.n_force + 1); f_hi = bq; }
    else if ((q + 1) % d.ratio != 0) { f_lo = bq; f_hi = bq; }
    else { f_lo = 1; f_hi = 0; }
}

constexpr int HBINS = 4096;      // histogram bins of one selection level (12 key bits)
constexpr int CAND_MAX = 1024;   // threshold-bin candidates ranked directly

struct SelSmem {
    typedef cub::BlockScan<int, SEL_THREADS> Scan;
    typename Scan::TempStorage scan;
    unsigned hist[HBINS];
    int cand[CAND_MAX];
    int ncand;
    int nkept;
    int bcast[4];
};

// Selection of the query at q by the whole CTA over its scores `sc` (shared memory), writing the
// ascending block list.  Keys are the bit patterns of the non-negative scores (order-preserving).
// Threshold search: histograms of 12 key bits ([30:19], then [18:7], then [6:0]) locate the bin
// holding the cut and how many of its keys to keep; once that bin holds at most CAND_MAX keys
// they are ranked directly (score, then lower block index).  Keys above the bin are kept.
// Sharded mode (cand_scores != null): only blocks in [blo, bhi) compete, forced blocks are left
// to the global merge, and each kept block's score is written beside it.
// The kept candidates kept[0..nk) (any order) written in ascending block order, then (unless
// sharded) the forced blocks f_lo.. (above every candidate); the list is padded as the
// compaction pads it.
__device__ void emit_kept(const DevDesc & d, const int * kept, int nk, int f_lo, int n_forced,
                          const float * __restrict__ sc, int * __restrict__ sel, int * __restrict__ nsel_out,
                          int * __restrict__ sel_out, bool shard, float * __restrict__ cand_scores) {
    const int tid = threadIdx.x;
    for (int i = tid; i < nk; i += blockDim.x) {
        const int bi = kept[i];
        int pos = 0;
        for (int j = 0; j < nk; j++) pos += kept[j] < bi;
        if (pos < d.kb) {
            sel[pos] = bi;
            if (sel_out) sel_out[pos] = bi;
            if (shard) cand_scores[pos] = sc[bi];
        }
    }
    int total = nk;
    if (!shard) {
        for (int i = tid; i < n_forced; i += blockDim.x) {
            const int pos = nk + i;
            if (pos < d.kb) {
                sel[pos] = f_lo + i;
                if (sel_out) sel_out[pos] = f_lo + i;
            }
        }
        total += n_forced;
    }
    const int n = min(total, d.kb);
    for (int i = n + tid; i < d.kb; i += blockDim.x) {
        if (sel_out) sel_out[i] = -1;
        if (shard) { sel[i] = -1; cand_scores[i] = 0.0f; }
    }
    if (tid == 0) *nsel_out = n;
}

// pre != null: the caller's load of the scores already cleared the candidates' flags and left in
// pre[0..2] this thread's count, smallest and largest positive candidate key.
__device__ void select_blocks(const DevDesc & d, int q, const float * __restrict__ sc, unsigned char * __restrict__ flag,
                              int * __restrict__ sel, int * __restrict__ nsel_out, int * __restrict__ sel_out,
                              SelSmem & sm, int blo, int bhi, float * __restrict__ cand_scores,
                              const uint32_t * pre = nullptr) {
    const bool shard = cand_scores != nullptr;
    const int tid = threadIdx.x;
    const int n_vis = (q + 1) / d.ratio;
    int f_lo, f_hi;
    forced_range(d, q, f_lo, f_hi);
    const int n_forced = f_hi >= f_lo ? f_hi - f_lo + 1 : 0;
    const int want = max(0, d.kb - n_forced);
    const int lo_c = max(blo, 0), hi_c = min(bhi, n_vis);          // candidate range
    const int n_cand = max(0, hi_c - lo_c) - max(0, min(f_hi, hi_c - 1) - max(f_lo, lo_c) + 1);
    auto is_cand = [&](int b) { return b >= lo_c && b < hi_c && !(b >= f_lo && b <= f_hi); };
    // The forced blocks are the top of the visible range, so the candidates are one run [lo_c, c_end)
    const int c_end = max(lo_c, n_forced ? min(hi_c, f_lo) : hi_c);
    const bool take_all = n_cand <= want;
    uint32_t prefix = 0, pmask = 0;   // keys with (key & pmask) > prefix are kept
    int remaining = 0;                // keys with (key & pmask) == prefix to keep
    bool ranked = false;              // the bin's keys were ranked into flag[]
    if (!pre)
        for (int b = tid; b < n_vis; b += blockDim.x) flag[b] = 0;
    if (!take_all) {
        remaining = want;
        // Zero scores (relu cut every head) can only fill what the positive ones leave: count the
        // positive candidates; when they are too few the cut is at 0 and zeros go by lowest index.
        // The same pass finds the smallest and largest positive key: the bits they share are shared
        // by every positive key, so the histogram levels start at the highest differing bit.
        int n_pos = 0;
        uint32_t kmin = 0xffffffffu, kmax = 0u;
        if (pre) {
            n_pos = (int) pre[0]; kmin = pre[1]; kmax = pre[2];
        } else {
            for (int b = lo_c + tid; b < c_end; b += blockDim.x) {
                const uint32_t key = __float_as_uint(sc[b]);
                if (key != 0u) { n_pos++; kmin = min(kmin, key); kmax = max(kmax, key); }
            }
        }
        #pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            n_pos += __shfl_xor_sync(0xffffffffu, n_pos, o);
            kmin = min(kmin, __shfl_xor_sync(0xffffffffu, kmin, o));
            kmax = max(kmax, __shfl_xor_sync(0xffffffffu, kmax, o));
        }
        const int nwarps = (int) (blockDim.x >> 5);
        if ((tid & 31) == 0) {
            sm.hist[tid >> 5] = (unsigned) n_pos;
            sm.hist[nwarps + (tid >> 5)] = kmin;
            sm.hist[2 * nwarps + (tid >> 5)] = kmax;
        }
        __syncthreads();
        if (tid == 0) {
            int tot = 0;
            uint32_t mn = 0xffffffffu, mx = 0u;
            for (int w = 0; w < nwarps; w++) {
                tot += (int) sm.hist[w];
                mn = min(mn, sm.hist[nwarps + w]);
                mx = max(mx, sm.hist[2 * nwarps + w]);
            }
            sm.bcast[3] = tot;
            sm.bcast[0] = (int) mn;
            sm.bcast[1] = (int) mx;
        }
        __syncthreads();
        n_pos = sm.bcast[3];
        kmin = (uint32_t) sm.bcast[0];
        kmax = (uint32_t) sm.bcast[1];
        __syncthreads();
        if (n_pos < remaining) {               // cut at zero: every positive key is kept
            prefix = 0; pmask = 0xffffffffu; remaining -= n_pos;
            goto compaction;
        }
        if (kmin == kmax) {                    // every positive key equal: the first `remaining` by index
            prefix = kmax; pmask = 0xffffffffu;
            goto compaction;
        }
        int hb = 31 - __clz(kmin ^ kmax);      // bits above hb are common to every positive key
        pmask = ~((2u << hb) - 1u);
        prefix = kmax & pmask;
        while (hb >= 0) {
            const int width = min(12, hb + 1), shift = hb + 1 - width, nb = 1 << width;
            hb = shift - 1;
            const uint32_t bmask = (uint32_t) (nb - 1);
            for (int i = tid; i < nb; i += blockDim.x) sm.hist[i] = 0;
            __syncthreads();
            for (int b = lo_c + tid; b < c_end; b += blockDim.x) {
                const uint32_t key = __float_as_uint(sc[b]);
                if (key != 0u && (key & pmask) == prefix) atomicAdd(&sm.hist[(key >> shift) & bmask], 1u);
            }
            __syncthreads();
            // thread i owns bins counted from the top: [nb - per*(i+1), nb - per*i)
            const int per = (nb + SEL_THREADS - 1) / SEL_THREADS;
            const int hi_bin = nb - per * tid;
            int own = 0;
            for (int k = 0; k < per; k++) {
                const int bin = hi_bin - 1 - k;
                if (bin >= 0) own += (int) sm.hist[bin];
            }
            int above;
            SelSmem::Scan(sm.scan).ExclusiveSum(own, above);
            if (above < remaining && above + own >= remaining) {        // exactly one thread
                int cum = above, bin = hi_bin - 1;
                for (int k = 0; k < per; k++, bin--) {
                    const int h = (int) sm.hist[bin];
                    if (cum + h >= remaining) break;
                    cum += h;
                }
                sm.bcast[0] = bin;
                sm.bcast[1] = remaining - cum;
                sm.bcast[2] = (int) sm.hist[bin];
            }
            __syncthreads();
            prefix |= (uint32_t) sm.bcast[0] << shift;
            pmask |= bmask << shift;
            remaining = sm.bcast[1];
            const int in_bin = sm.bcast[2];
            __syncthreads();
            if (in_bin <= CAND_MAX) {
                // One pass collects the keys above the cut bin (kept) and the bin's keys, which are
                // ranked directly (score, then lower block); the kept list (at most kb) is then put
                // in block order without another pass over the scores.
                int * kept = reinterpret_cast<int *>(sm.hist);
                if (tid == 0) { sm.ncand = 0; sm.nkept = 0; }
                __syncthreads();
                for (int b = lo_c + tid; b < c_end; b += blockDim.x) {
                    const uint32_t key = __float_as_uint(sc[b]);
                    if (key == 0u) continue;
                    const uint32_t km = key & pmask;
                    if (km > prefix) {
                        const int slot = atomicAdd(&sm.nkept, 1);
                        if (slot < MAX_KB) kept[slot] = b;
                    } else if (km == prefix) {
                        const int slot = atomicAdd(&sm.ncand, 1);
                        if (slot < CAND_MAX) sm.cand[slot] = b;
                    }
                }
                __syncthreads();
                const int m = min(sm.ncand, CAND_MAX);
                for (int i = tid; i < m; i += blockDim.x) {
                    const int bi = sm.cand[i];
                    const uint32_t ki = __float_as_uint(sc[bi]);
                    int rank = 0;
                    for (int jx = 0; jx < m; jx++) {
                        const int bj = sm.cand[jx];
                        const uint32_t kj = __float_as_uint(sc[bj]);
                        rank += (kj > ki) || (kj == ki && bj < bi);
                    }
                    if (rank < remaining) {
                        const int slot = atomicAdd(&sm.nkept, 1);
                        if (slot < MAX_KB) kept[slot] = bi;
                    }
                }
                __syncthreads();
                emit_kept(d, kept, min(sm.nkept, MAX_KB), f_lo, n_forced, sc, sel, nsel_out, sel_out, shard, cand_scores);
                return;
            }
        }
        __syncthreads();
    }
compaction:
    // Compaction over [0, max(n_vis, f_hi+1)) in ascending order: each thread owns a contiguous run.
    // Without ranking (more than CAND_MAX equal keys) the bin's first `remaining` by index are kept,
    // which needs the number of such ties before each thread's run.
    const int r_lo = shard ? lo_c : 0, r_hi = shard ? max(lo_c, hi_c) : max(n_vis, f_hi + 1);
    const int per = (r_hi - r_lo + blockDim.x - 1) / blockDim.x;
    const int lo = r_lo + tid * per, hi = min(r_hi, lo + per);
    const bool tie_quota = !take_all && !ranked;
    int tie_base = 0;
    if (tie_quota) {
        int n_tie = 0;
        for (int b = lo; b < hi; b++)
            if (is_cand(b) && (__float_as_uint(sc[b]) & pmask) == prefix) n_tie++;
        SelSmem::Scan(sm.scan).ExclusiveSum(n_tie, tie_base);
        __syncthreads();
    }
    auto take = [&](int b, int & tie_i) -> bool {
        if (b >= f_lo && b <= f_hi) return !shard;
        if (!is_cand(b)) return false;
        if (take_all) return true;
        const uint32_t km = __float_as_uint(sc[b]) & pmask;
        if (km > prefix) return true;
        if (km != prefix) return false;
        if (ranked) return flag[b] != 0;
        return tie_i++ < remaining;
    };
    unsigned long long bits = 0;                       // take flags of the run (runs of <= 64)
    int n_take = 0, tie_i = tie_base;
    for (int b = lo; b < hi; b++) {
        const bool tk = take(b, tie_i);
        n_take += tk;
        if (per <= 64 && tk) bits |= 1ull << (b - lo);
    }
    int base, total;
    SelSmem::Scan(sm.scan).ExclusiveSum(n_take, base, total);
    int pos = base;
    if (per <= 64) {
        while (bits) {
            const int b = lo + __ffsll((long long) bits) - 1;
            bits &= bits - 1;
            if (pos < d.kb) {
                sel[pos] = b;
                if (sel_out) sel_out[pos] = b;
                if (shard) cand_scores[pos] = sc[b];
            }
            pos++;
        }
    } else {
        tie_i = tie_base;
        for (int b = lo; b < hi; b++) {
            if (take(b, tie_i)) {
                if (pos < d.kb) {
                    sel[pos] = b;
                    if (sel_out) sel_out[pos] = b;
                    if (shard) cand_scores[pos] = sc[b];
                }
                pos++;
            }
        }
    }
    const int n = min(total, d.kb);
    for (int i = n + tid; i < d.kb; i += blockDim.x) {
        if (sel_out) sel_out[i] = -1;
        if (shard) { sel[i] = -1; cand_scores[i] = 0.0f; }
    }
    if (tid == 0) *nsel_out = n;
}

// grid = (score CTAs per query, n_queries).  Query t: position q_pos(t), pooled cache `pool`.
// Decode: items != null (per-query caches and n_past); prefill: one cache, q = n_past0 + t.
// Replicated indexer caches: the global selection stays in sel_out; the attention's list keeps the
// blocks of this shard's K/V rows, in order.
__device__ void keep_shard_blocks(const DevDesc & d, int * __restrict__ list, int * __restrict__ nsel, SelSmem & sm) {
    __syncthreads();                                 // the selection's stores are visible to the CTA
    const int n = *nsel;
    const int i = threadIdx.x;
    const int b = i < n && i < d.kb ? list[i] : -1;
    const bool keep = b >= d.shard_blk0 && b < d.shard_blk1;
    int rank;
    SelSmem::Scan(sm.scan).ExclusiveSum(keep ? 1 : 0, rank);
    __syncthreads();                                 // every thread has read its entry
    if (keep) list[rank] = b;
    if (i == SEL_THREADS - 1) sm.bcast[0] = rank + (keep ? 1 : 0);
    __syncthreads();
    const int m = sm.bcast[0];
    for (int j = m + i; j < d.kb; j += SEL_THREADS) list[j] = -1;
    if (i == 0) *nsel = m;
}

__global__ void __launch_bounds__(SEL_THREADS) score_select_kernel(DevDesc d,
        const qsa_decode_item * __restrict__ items, const uint16_t * __restrict__ pool0, int n_past0,
        const float * __restrict__ q_idx, int blocks_per_cta,
        float * __restrict__ scores_ws, int scores_stride, unsigned * __restrict__ counters,
        int * __restrict__ sel_ws, int * __restrict__ nsel_ws, int * __restrict__ sel_out,
        uint32_t * __restrict__ status, float * __restrict__ cand_scores) {
    extern __shared__ __align__(16) unsigned char dyn_smem[];
    __shared__ SelSmem sm;
    __shared__ bool is_last;
    pdl_trigger();
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

    // Decode with a window: this step's append writes only the query's own block (its pooled
    // key included), which is forced, so scoring need not wait for it; the wait moves to the exit
    // (the attention, launched behind this grid, still finds the appended row).
    const bool defer_wait = items != nullptr && d.window > 0;
    if (!bad) {
        float qf[4][8];
        const int sub = threadIdx.x & 15;
        #pragma unroll
        for (int h = 0; h < 4; h++)
            #pragma unroll
            for (int e = 0; e < 8; e++)
                qf[h][e] = h < d.idx_n_head
                    ? f16_bits_to_f32(f32_to_f16_bits(q_idx[((size_t) t * d.idx_n_head + h) * d.idx_dim + 8 * sub + e]))
                    : 0.0f;
        // candidates only: the forced blocks are the top of the visible range and never compete
        int f_lo, f_hi;
        forced_range(d, q, f_lo, f_hi);
        const int cand_hi = f_lo <= f_hi ? min(n_vis, f_lo) : n_vis;
        const int b0 = blo + blockIdx.x * blocks_per_cta;
        const int b1 = min(min(cand_hi, bhi), b0 + blocks_per_cta);
        if (!defer_wait) pdl_wait();             // the append of this step (pooled keys) is complete
        if (b0 < b1) score_range(d, pool, qf, b0, b1, sc);
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
    if (!is_last) {
        if (defer_wait) pdl_wait();
        return;
    }
    float * ssc = reinterpret_cast<float *>(dyn_smem);
    unsigned char * flag = dyn_smem + (size_t) scores_stride * 4;
    uint32_t pre[3] = {0u, 0xffffffffu, 0u};       // this thread's count, min and max positive candidate key
    {   // the query's scores in [blo, n_vis), 16 bytes per load (score rows are 16-byte aligned); the
        // same loop clears the candidates' selection flags and gathers what the selection's first
        // pass needs
        int f_lo, f_hi;
        forced_range(d, q, f_lo, f_hi);
        const int lo_c = max(blo, 0), hi_c = min(bhi, n_vis);
        const int c_end = max(lo_c, f_lo <= f_hi ? min(hi_c, f_lo) : hi_c);   // candidates [lo_c, c_end)
        const int i0 = max(blo, 0) / 4, n4 = (min(n_vis, bhi) + 3) / 4;
        #pragma unroll 4
        for (int i = i0 + threadIdx.x; i < n4; i += blockDim.x) {
            const float4 v = __ldcg(reinterpret_cast<const float4 *>(sc) + i);
            reinterpret_cast<float4 *>(ssc)[i] = v;
            reinterpret_cast<uint32_t *>(flag)[i] = 0u;
            const float e[4] = {v.x, v.y, v.z, v.w};
            #pragma unroll
            for (int k = 0; k < 4; k++) {
                const int b = 4 * i + k;
                const uint32_t key = __float_as_uint(e[k]);
                if (b >= lo_c && b < c_end && key != 0u) {
                    pre[0]++;
                    pre[1] = min(pre[1], key);
                    pre[2] = max(pre[2], key);
                }
            }
        }
    }
    __syncthreads();
    if (bad) {
        for (int i = threadIdx.x; i < d.kb; i += blockDim.x) {
            sel_ws[(size_t) t * d.kb + i] = -1;
            if (sel_out) sel_out[(size_t) t * d.kb + i] = -1;
            if (cand_scores) cand_scores[(size_t) t * d.kb + i] = 0.0f;
        }
        if (threadIdx.x == 0) nsel_ws[t] = 0;
        if (defer_wait) pdl_wait();
        return;
    }
    select_blocks(d, q, ssc, flag, sel_ws + (size_t) t * d.kb, nsel_ws + t,
                  sel_out ? sel_out + (size_t) t * d.kb : nullptr, sm, blo, bhi,
                  cand_scores ? cand_scores + (size_t) t * d.kb : nullptr, pre);
    if (d.shard_ri) keep_shard_blocks(d, sel_ws + (size_t) t * d.kb, nsel_ws + t, sm);
    if (defer_wait) pdl_wait();                  // the append is complete before this grid is
}

}  // namespace qsa
