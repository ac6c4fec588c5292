// qsa_shard.cu -- the exchange steps of KV-sequence-sharded decode.
//
// The reference runs on one device (README.md:215); sharding the KV sequence axis across GPUs is
// this library's addition for very long contexts.  Rank g owns blocks [blo, bhi) of every layer.
// One step: every rank scores its blocks and keeps its local best (score_select_kernel in sharded
// mode); the candidates of all ranks are all-gathered by the caller; shard_select_kernel forms
// the exact global selection on every rank (every global winner is in its owner's local best;
// a radix select over the gathered scores, one warp per query);
// each rank attends its own selected blocks into an unnormalised state (attn_kernel, state mode);
// the states are all-gathered and merge_states_kernel combines them by log-sum-exp in rank order.
#include "qsa_kernels.cuh"

namespace qsa {

constexpr int SHARD_SEL_WARPS = 8;        // queries per CTA (one warp each)

// Forced blocks of the query at q (the same rule as the selection kernel).
__device__ __forceinline__ void shard_forced_range(const DevDesc & d, int q, int & f_lo, int & f_hi) {
    const int bq = q / d.ratio;
    if (d.window > 0) { f_lo = max(0, bq - d.n_force + 1); f_hi = bq; }
    else if ((q + 1) % d.ratio != 0) { f_lo = bq; f_hi = bq; }
    else { f_lo = 1; f_hi = 0; }
}

__device__ __forceinline__ int warp_incl_scan(int x, int lane) {
    #pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, x, o);
        if (lane >= o) x += y;
    }
    return x;
}

// One warp per query.  Candidates: per shard (cand_stride int32 apart) int32 [2][batch][kb], the
// block ids (-1 = none), then the f32 scores' bits.  Every shard sends its kept blocks in
// ascending order and the shards hold ascending block ranges, so the concatenation of the lists
// (slot order) is ascending by block: a radix select over the scores (8-bit digits from the top)
// with the lower slot first on equal scores is the global rule (score, then lower block).  Writes
// the global selection (ascending, -1 padded) to sel_out (optional) and this rank's blocks
// [blo, bhi) of it to the workspace list the attention kernel reads.  A candidate that no shard
// could have sent (not visible, forced, or not a non-negative score) is dropped and flagged.
__global__ void __launch_bounds__(32 * SHARD_SEL_WARPS) shard_select_kernel(DevDesc d,
        const qsa_decode_item * __restrict__ items, int n_shards, int batch,
        const int * __restrict__ cand, size_t cand_stride, int blo, int bhi,
        int * __restrict__ sel_out, int * __restrict__ sel_ws, int * __restrict__ nsel_ws,
        uint32_t * __restrict__ status) {
    __shared__ unsigned hist[SHARD_SEL_WARPS][256];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int t = blockIdx.x * SHARD_SEL_WARPS + warp;
    if (t >= batch) return;
    const int q = items[t].n_past;
    const int kb = d.kb;
    int * sw = sel_ws + (size_t) t * kb;
    int * so = sel_out ? sel_out + (size_t) t * kb : nullptr;
    if (q < 0 || q >= d.n_ctx) {
        if (lane == 0) { set_status(status, DEV_BAD_POS); nsel_ws[t] = 0; }
        for (int i = lane; i < kb; i += 32) { sw[i] = -1; if (so) so[i] = -1; }
        return;
    }
    int f_lo, f_hi;
    shard_forced_range(d, q, f_lo, f_hi);
    const int n_forced = f_hi >= f_lo ? f_hi - f_lo + 1 : 0;
    const int want = max(0, kb - n_forced);
    const int n_vis = (q + 1) / d.ratio;
    const int n = n_shards * kb;                     // candidate slots, slot i = shard i / kb, entry i % kb
    auto slot_block = [&](int i) -> int {
        return cand[(size_t) (i / kb) * cand_stride + (size_t) t * kb + (i % kb)];
    };
    auto slot_key = [&](int i) -> uint32_t {
        return (uint32_t) cand[(size_t) (i / kb) * cand_stride + (size_t) (batch + t) * kb + (i % kb)];
    };
    auto valid = [&](int b, uint32_t key) {
        return b >= 0 && b < n_vis && !(b >= f_lo && b <= f_hi) && (key >> 31) == 0u && key <= 0x7f800000u;
    };
    const int per = (n + 31) / 32;
    const int lo = min(n, lane * per), hi = min(n, lo + per);
    int n_valid = 0;
    for (int i = lo; i < hi; i++) {
        const int b = slot_block(i);
        if (b < 0) continue;
        if (valid(b, slot_key(i))) n_valid++;
        else set_status(status, DEV_BAD_SEL);
    }
    int tot_valid = warp_incl_scan(n_valid, lane);
    tot_valid = __shfl_sync(0xffffffffu, tot_valid, 31);
    const bool take_all = tot_valid <= want;
    uint32_t prefix = 0, pmask = 0;
    int remaining = want;
    unsigned * hw = hist[warp];
    if (!take_all && want > 0) {
        for (int shift = 24; shift >= 0; shift -= 8) {
            for (int i = lane; i < 256; i += 32) hw[i] = 0;
            __syncwarp();
            for (int i = lo; i < hi; i++) {
                const int b = slot_block(i);
                const uint32_t key = slot_key(i);
                if (valid(b, key) && (key & pmask) == prefix) atomicAdd(&hw[(key >> shift) & 255u], 1u);
            }
            __syncwarp();
            int own = 0;
            #pragma unroll
            for (int k = 0; k < 8; k++) own += (int) hw[255 - 8 * lane - k];
            const int incl = warp_incl_scan(own, lane);
            const int above = incl - own;
            const unsigned hit = __ballot_sync(0xffffffffu, above < remaining && incl >= remaining);
            const int src = __ffs(hit) - 1;
            int bin = 0, cut_rem = 0;
            if (lane == src) {
                int cum = above, k = 0;
                for (; k < 8; k++) {
                    const int hc = (int) hw[255 - 8 * lane - k];
                    if (cum + hc >= remaining) break;
                    cum += hc;
                }
                bin = 255 - 8 * lane - k;
                cut_rem = remaining - cum;
            }
            bin = __shfl_sync(0xffffffffu, bin, src);
            cut_rem = __shfl_sync(0xffffffffu, cut_rem, src);
            prefix |= (uint32_t) bin << shift;
            pmask |= 255u << shift;
            remaining = cut_rem;
            __syncwarp();
        }
    }
    const bool none = !take_all && want == 0;
    // per slot: 2 kept, 1 equal to the cut, 0 not kept
    auto cls = [&](int i) -> int {
        const int b = slot_block(i);
        const uint32_t key = slot_key(i);
        if (!valid(b, key) || none) return 0;
        if (take_all) return 2;
        return key > prefix ? 2 : (key == prefix ? 1 : 0);
    };
    int n_take = 0, n_tie = 0;
    for (int i = lo; i < hi; i++) {
        const int c = cls(i);
        n_take += c == 2;
        n_tie += c == 1;
    }
    const int tie_incl = warp_incl_scan(n_tie, lane);
    const int tie_mine = max(0, min(n_tie, remaining - (tie_incl - n_tie)));
    // positions in the global list and in this rank's list
    int n_mine_rank = 0;
    {
        int tl = tie_mine;
        for (int i = lo; i < hi; i++) {
            const int c = cls(i);
            bool tk = c == 2;
            if (c == 1 && tl > 0) { tk = true; tl--; }
            if (tk) { const int b = slot_block(i); n_mine_rank += b >= blo && b < bhi; }
        }
    }
    const int mine = n_take + tie_mine;
    const int pos_incl = warp_incl_scan(mine, lane), rk_incl = warp_incl_scan(n_mine_rank, lane);
    int pos = pos_incl - mine, rpos = rk_incl - n_mine_rank;
    const int n_cand_kept = __shfl_sync(0xffffffffu, pos_incl, 31);
    const int n_rank_kept = __shfl_sync(0xffffffffu, rk_incl, 31);
    int tl = tie_mine;
    for (int i = lo; i < hi; i++) {
        const int c = cls(i);
        bool tk = c == 2;
        if (c == 1 && tl > 0) { tk = true; tl--; }
        if (!tk) continue;
        const int b = slot_block(i);
        if (so && pos < kb) so[pos] = b;
        pos++;
        if (b >= blo && b < bhi) { if (rpos < kb) sw[rpos] = b; rpos++; }
    }
    // the forced blocks follow (they are above every candidate)
    const int f_rank_lo = max(f_lo, blo), f_rank_hi = min(f_hi, bhi - 1);
    const int n_f_rank = n_forced ? max(0, f_rank_hi - f_rank_lo + 1) : 0;
    for (int i = lane; i < n_forced; i += 32) {
        if (so && n_cand_kept + i < kb) so[n_cand_kept + i] = f_lo + i;
    }
    for (int i = lane; i < n_f_rank; i += 32) {
        if (n_rank_kept + i < kb) sw[n_rank_kept + i] = f_rank_lo + i;
    }
    const int m_all = min(kb, n_cand_kept + n_forced), m_rank = min(kb, n_rank_kept + n_f_rank);
    if (so) for (int i = m_all + lane; i < kb; i += 32) so[i] = -1;
    for (int i = m_rank + lane; i < kb; i += 32) sw[i] = -1;
    if (lane == 0) nsel_ws[t] = m_rank;
}

// out[t][h][d] from the gathered states [n_parts][batch][M 16 | L 16 | O 16x256], merged in rank
// order: M = max_p m_p, out = sum_p 2^(m_p - M) O_p / sum_p 2^(m_p - M) l_p.
__global__ void __launch_bounds__(256) merge_states_kernel(DevDesc d, int n_parts, int batch,
        const float * __restrict__ states, float * __restrict__ out) {
    constexpr int ROWS = 16, SF = 2 * ROWS + ROWS * HEAD_DIM;
    const int t = blockIdx.x, hr = blockIdx.y, dim = threadIdx.x;
    const int g = hr >> 3, h = hr & 7;
    if (g >= d.n_head_kv || h >= d.gqa) return;
    float M = -INFINITY;
    for (int p = 0; p < n_parts; p++) M = fmaxf(M, states[((size_t) p * batch + t) * SF + hr]);
    const float Mu = M == -INFINITY ? 0.0f : M;
    float L = 0.0f, acc = 0.0f;
    for (int p = 0; p < n_parts; p++) {
        const float * st = states + ((size_t) p * batch + t) * SF;
        const float w = exp2f(st[hr] - Mu);
        L += st[ROWS + hr] * w;
        acc += st[2 * ROWS + hr * HEAD_DIM + dim] * w;
    }
    out[((size_t) t * d.n_head + g * d.gqa + h) * HEAD_DIM + dim] = L > 0.0f ? acc / L : 0.0f;
}

cudaError_t launch_shard_select(const DevDesc & d, cudaStream_t st, const qsa_decode_item * items, int n_shards,
        int batch, const int * cand, size_t cand_stride, int blo, int bhi, int * sel_out, int * sel_ws, int * nsel_ws,
        uint32_t * status) {
    shard_select_kernel<<<(batch + SHARD_SEL_WARPS - 1) / SHARD_SEL_WARPS, 32 * SHARD_SEL_WARPS, 0, st>>>(
        d, items, n_shards, batch, cand, cand_stride, blo, bhi, sel_out, sel_ws, nsel_ws, status);
    return cudaGetLastError();
}

cudaError_t launch_merge_states(const DevDesc & d, cudaStream_t st, int n_parts, int batch, const float * states,
                                float * out) {
    merge_states_kernel<<<dim3(batch, 16), HEAD_DIM, 0, st>>>(d, n_parts, batch, states, out);
    return cudaGetLastError();
}

}  // namespace qsa
