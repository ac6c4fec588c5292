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
// With the indexer caches replicated every rank selects globally itself, and the fused peer
// exchange has the attention store the states into every rank's region; merge_states_kernel then
// waits for the ranks' flags before it reads them.
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
// with the lower slot first on equal scores is the global rule (score, then lower block).  The
// warp stages its query's slots in shared memory (coalesced), runs the radix passes over them and
// emits the kept slots 32 at a time in slot order with ballots.  Writes the global selection
// (ascending, -1 padded) to sel_out (optional) and this rank's blocks [blo, bhi) of it to the
// workspace list the attention kernel reads.  A candidate that no shard could have sent (not
// visible, forced, or not a non-negative score) is dropped and flagged.
__global__ void shard_select_kernel(DevDesc d, const qsa_decode_item * __restrict__ items, int n_shards, int batch,
        const int * __restrict__ cand, size_t cand_stride, int blo, int bhi,
        int * __restrict__ sel_out, int * __restrict__ sel_ws, int * __restrict__ nsel_ws,
        uint32_t * __restrict__ status) {
    extern __shared__ int ss_smem[];                 // per warp: [n] block ids, then [n] keys
    __shared__ unsigned hist[SHARD_SEL_WARPS][256];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int t = blockIdx.x * (blockDim.x >> 5) + warp;
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
    int * sb = ss_smem + (size_t) warp * 2 * n;
    uint32_t * sk = reinterpret_cast<uint32_t *>(sb + n);
    int n_valid = 0;
    for (int s = 0; s < n_shards; s++) {
        const int * ids = cand + (size_t) s * cand_stride + (size_t) t * kb;
        const int * keys = cand + (size_t) s * cand_stride + (size_t) (batch + t) * kb;
        for (int j = lane; j < kb; j += 32) {
            int b = ids[j];
            const uint32_t key = (uint32_t) keys[j];
            if (b >= 0) {
                if (b < n_vis && !(b >= f_lo && b <= f_hi) && (key >> 31) == 0u && key <= 0x7f800000u) n_valid++;
                else { set_status(status, DEV_BAD_SEL); b = -1; }
            }
            sb[s * kb + j] = b;
            sk[s * kb + j] = key;
        }
    }
    __syncwarp();
    int tot_valid = warp_incl_scan(n_valid, lane);
    tot_valid = __shfl_sync(0xffffffffu, tot_valid, 31);
    const bool take_all = tot_valid <= want;
    uint32_t prefix = 0, pmask = 0;
    int remaining = want;
    unsigned * hw = hist[warp];
    if (!take_all && want > 0) {
        // the bits every valid key shares need no pass: digits start at the highest differing bit
        uint32_t kmin = 0xffffffffu, kmax = 0u;
        for (int i = lane; i < n; i += 32)
            if (sb[i] >= 0) { kmin = min(kmin, sk[i]); kmax = max(kmax, sk[i]); }
        #pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            kmin = min(kmin, __shfl_xor_sync(0xffffffffu, kmin, o));
            kmax = max(kmax, __shfl_xor_sync(0xffffffffu, kmax, o));
        }
        int hi_bit = kmin == kmax ? -1 : 31 - __clz(kmin ^ kmax);
        // bits 0..hi_bit (none when every valid key is equal: the cut is that key)
        const uint32_t low = hi_bit < 0 ? 0u : (hi_bit >= 31 ? 0xffffffffu : (2u << hi_bit) - 1u);
        pmask = ~low;
        prefix = kmax & pmask;
        while (hi_bit >= 0) {
            const int width = min(8, hi_bit + 1), shift = hi_bit + 1 - width;
            const uint32_t dmask = (1u << width) - 1u;
            for (int i = lane; i < 256; i += 32) hw[i] = 0;
            __syncwarp();
            for (int i = lane; i < n; i += 32)
                if (sb[i] >= 0 && (sk[i] & pmask) == prefix) atomicAdd(&hw[(sk[i] >> shift) & dmask], 1u);
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
            pmask |= dmask << shift;
            remaining = cut_rem;
            hi_bit = shift - 1;
            __syncwarp();
        }
    }
    const bool none = !take_all && want == 0;
    // emission in slot order: keys above the cut kept, keys equal to it by lower slot, `remaining`
    // of them; positions in the global list and in this rank's list by ballots
    const unsigned lt = (1u << lane) - 1u;
    int n_cand_kept = 0, n_rank_kept = 0, ties_seen = 0;
    for (int i0 = 0; i0 < n; i0 += 32) {
        const int i = i0 + lane;
        int c = 0, b = -1;
        if (i < n && !none) {
            b = sb[i];
            if (b >= 0) c = take_all ? 2 : (sk[i] > prefix ? 2 : (sk[i] == prefix ? 1 : 0));
        }
        const unsigned tieb = __ballot_sync(0xffffffffu, c == 1);
        const bool tk = c == 2 || (c == 1 && ties_seen + __popc(tieb & lt) < remaining);
        const unsigned tb = __ballot_sync(0xffffffffu, tk);
        const bool rk = tk && b >= blo && b < bhi;
        const unsigned rb = __ballot_sync(0xffffffffu, rk);
        const int pos = n_cand_kept + __popc(tb & lt), rpos = n_rank_kept + __popc(rb & lt);
        if (tk && so && pos < kb) so[pos] = b;
        if (rk && rpos < kb) sw[rpos] = b;
        n_cand_kept += __popc(tb);
        n_rank_kept += __popc(rb);
        ties_seen += __popc(tieb);
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

// The same selection for lists of up to SORT_MAX slots, one CTA per query: each slot's 64-bit key
// (score bits, then the complement of its slot index; 0 for an empty or dropped slot) is sorted
// descending by a bitonic network in shared memory, so the first `want` keys are the kept ones
// (higher score, then lower block); kept flags are then scanned in slot order (ascending blocks).
constexpr int SORT_MAX = 2048;

__global__ void __launch_bounds__(1024) shard_select_sort_kernel(DevDesc d, const qsa_decode_item * __restrict__ items,
        int n_shards, int batch, const int * __restrict__ cand, size_t cand_stride, int blo, int bhi,
        int * __restrict__ sel_out, int * __restrict__ sel_ws, int * __restrict__ nsel_ws, uint32_t * __restrict__ status) {
    __shared__ unsigned long long key[SORT_MAX];
    __shared__ int blk[SORT_MAX];
    __shared__ unsigned char kept[SORT_MAX];
    __shared__ int wsum[2][32];
    __shared__ int n_valid_s;
    const int t = blockIdx.x, tid = threadIdx.x, nthr = blockDim.x, lane = tid & 31, warp = tid >> 5;
    const int q = items[t].n_past;
    const int kb = d.kb;
    int * sw = sel_ws + (size_t) t * kb;
    int * so = sel_out ? sel_out + (size_t) t * kb : nullptr;
    if (q < 0 || q >= d.n_ctx) {
        if (tid == 0) { set_status(status, DEV_BAD_POS); nsel_ws[t] = 0; }
        for (int i = tid; i < kb; i += nthr) { sw[i] = -1; if (so) so[i] = -1; }
        return;
    }
    int f_lo, f_hi;
    shard_forced_range(d, q, f_lo, f_hi);
    const int n_forced = f_hi >= f_lo ? f_hi - f_lo + 1 : 0;
    const int want = max(0, kb - n_forced);
    const int n_vis = (q + 1) / d.ratio;
    const int n = n_shards * kb;
    int n2 = 1;
    while (n2 < n) n2 <<= 1;
    if (tid == 0) n_valid_s = 0;
    __syncthreads();
    int my_valid = 0;
    for (int i = tid; i < n2; i += nthr) {
        unsigned long long k = 0ull;
        int b = -1;
        if (i < n) {
            const int s = i / kb, j = i - s * kb;
            b = cand[(size_t) s * cand_stride + (size_t) t * kb + j];
            const uint32_t kbits = (uint32_t) cand[(size_t) s * cand_stride + (size_t) (batch + t) * kb + j];
            if (b >= 0) {
                if (b < n_vis && !(b >= f_lo && b <= f_hi) && (kbits >> 31) == 0u && kbits <= 0x7f800000u) {
                    k = ((unsigned long long) kbits << 32) | (0xffffffffu - (uint32_t) i);
                    my_valid++;
                } else {
                    set_status(status, DEV_BAD_SEL);
                    b = -1;
                }
            }
        }
        key[i] = k;
        if (i < n) { blk[i] = b; kept[i] = 0; }
    }
    if (my_valid) atomicAdd(&n_valid_s, my_valid);
    __syncthreads();
    // bitonic sort, descending
    for (int size = 2; size <= n2; size <<= 1) {
        for (int stride = size >> 1; stride > 0; stride >>= 1) {
            for (int i = tid; i < n2 / 2; i += nthr) {
                const int lo = 2 * i - (i & (stride - 1));     // index with the stride bit clear
                const int hi = lo + stride;
                const bool desc = (lo & size) == 0;
                const unsigned long long a = key[lo], c = key[hi];
                if ((a < c) == desc) { key[lo] = c; key[hi] = a; }
            }
            __syncthreads();
        }
    }
    const int n_keep = min(want, n_valid_s);
    for (int i = tid; i < n_keep; i += nthr) kept[0xffffffffu - (uint32_t) (key[i] & 0xffffffffull)] = 1;
    __syncthreads();
    // positions in slot order: a CTA scan of the kept flags (all kept, and this rank's)
    int n_cand_kept = 0, n_rank_kept = 0;
    for (int base = 0; base < n; base += nthr) {
        const int i = base + tid;
        const bool tk = i < n && kept[i];
        const int b = tk ? blk[i] : -1;
        const bool rk = tk && b >= blo && b < bhi;
        const unsigned tb = __ballot_sync(0xffffffffu, tk), rb = __ballot_sync(0xffffffffu, rk);
        if (lane == 0) { wsum[0][warp] = __popc(tb); wsum[1][warp] = __popc(rb); }
        __syncthreads();
        int pre_t = 0, pre_r = 0, tot_t = 0, tot_r = 0;
        for (int w = 0; w < nthr / 32; w++) {
            if (w < warp) { pre_t += wsum[0][w]; pre_r += wsum[1][w]; }
            tot_t += wsum[0][w];
            tot_r += wsum[1][w];
        }
        const unsigned lt = (1u << lane) - 1u;
        const int pos = n_cand_kept + pre_t + __popc(tb & lt), rpos = n_rank_kept + pre_r + __popc(rb & lt);
        if (tk && so && pos < kb) so[pos] = b;
        if (rk && rpos < kb) sw[rpos] = b;
        n_cand_kept += tot_t;
        n_rank_kept += tot_r;
        __syncthreads();
    }
    // the forced blocks follow (they are above every candidate)
    const int f_rank_lo = max(f_lo, blo), f_rank_hi = min(f_hi, bhi - 1);
    const int n_f_rank = n_forced ? max(0, f_rank_hi - f_rank_lo + 1) : 0;
    for (int i = tid; i < n_forced; i += nthr)
        if (so && n_cand_kept + i < kb) so[n_cand_kept + i] = f_lo + i;
    for (int i = tid; i < n_f_rank; i += nthr)
        if (n_rank_kept + i < kb) sw[n_rank_kept + i] = f_rank_lo + i;
    const int m_all = min(kb, n_cand_kept + n_forced), m_rank = min(kb, n_rank_kept + n_f_rank);
    if (so) for (int i = m_all + tid; i < kb; i += nthr) so[i] = -1;
    for (int i = m_rank + tid; i < kb; i += nthr) sw[i] = -1;
    if (tid == 0) nsel_ws[t] = m_rank;
}

// out[t][h][d] from the gathered states [n_parts][batch][M 16 | L 16 | O 16x256], merged in rank
// order: M = max_p m_p, out = sum_p 2^(m_p - M) O_p / sum_p 2^(m_p - M) l_p.
// flags != null: the states were stored into this rank's region by every rank and published by
// flag; each CTA first waits (bounded by 2 s of %globaltimer, then DEV_TIMEOUT, so the context
// stays usable) until every flag has reached *epoch, and reads the states from L2.
__device__ __forceinline__ uint32_t ld_acquire_sys_u32(const uint32_t * p) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__global__ void __launch_bounds__(256) merge_states_kernel(DevDesc d, int n_parts, int batch,
        const float * states, float * __restrict__ out, const uint32_t * flags, const uint32_t * epoch,
        uint32_t * status) {
    constexpr int ROWS = 16, SF = 2 * ROWS + ROWS * HEAD_DIM;
    const int t = blockIdx.x, hr = blockIdx.y, dim = threadIdx.x;
    const int g = hr >> 3, h = hr & 7;
    if (g >= d.n_head_kv || h >= d.gqa) return;
    if (flags) {
        if ((int) threadIdx.x < n_parts) {
            const uint32_t e = *reinterpret_cast<const volatile uint32_t *>(epoch);
            const uint32_t * f = flags + threadIdx.x;
            // a flag at or past this round's epoch: the rank's states of this round have landed
            if ((int32_t) (ld_acquire_sys_u32(f) - e) < 0) {
                const uint64_t t0 = global_timer_ns();
                while ((int32_t) (ld_acquire_sys_u32(f) - e) < 0) {
                    if (global_timer_ns() - t0 > 2000000000ull) {
                        set_status(status, DEV_TIMEOUT);
                        break;
                    }
                }
            }
        }
        __syncthreads();
    }
    auto ld = [&](size_t i) { return flags ? __ldcg(states + i) : states[i]; };
    float M = -INFINITY;
    for (int p = 0; p < n_parts; p++) M = fmaxf(M, ld(((size_t) p * batch + t) * SF + hr));
    const float Mu = M == -INFINITY ? 0.0f : M;
    float L = 0.0f, acc = 0.0f;
    for (int p = 0; p < n_parts; p++) {
        const size_t st = ((size_t) p * batch + t) * SF;
        const float w = exp2f(ld(st + hr) - Mu);
        L += ld(st + ROWS + hr) * w;
        acc += ld(st + 2 * ROWS + (size_t) hr * HEAD_DIM + dim) * w;
    }
    out[((size_t) t * d.n_head + g * d.gqa + h) * HEAD_DIM + dim] = L > 0.0f ? acc / L : 0.0f;
}

cudaError_t launch_shard_select(const DevDesc & d, cudaStream_t st, const qsa_decode_item * items, int n_shards,
        int batch, const int * cand, size_t cand_stride, int blo, int bhi, int * sel_out, int * sel_ws, int * nsel_ws,
        uint32_t * status) {
    const int n = n_shards * d.kb;
    if (n <= SORT_MAX) {                    // a CTA per query: bitonic sort of the slot keys
        int n2 = 1;
        while (n2 < n) n2 <<= 1;
        const int thr = std::max(32, std::min(1024, n2 / 2));
        shard_select_sort_kernel<<<batch, thr, 0, st>>>(d, items, n_shards, batch, cand, cand_stride, blo, bhi, sel_out,
                                                      sel_ws, nsel_ws, status);
        return cudaGetLastError();
    }
    // longer lists: a warp per query stages its slots (8 bytes each) in shared memory
    const size_t per_warp = (size_t) n * 8;
    constexpr size_t SMEM_MAX = 200 * 1024;
    if (per_warp > SMEM_MAX) return cudaErrorInvalidValue;
    const int warps = (int) std::min<size_t>(std::min<size_t>(SHARD_SEL_WARPS, SMEM_MAX / per_warp), (size_t) batch);
    const size_t smem = per_warp * warps;
    static std::atomic<uint64_t> attr{0};
    if (smem > 48 * 1024) {
        const cudaError_t e = once_per_device(attr, [] {
            return cudaFuncSetAttribute(shard_select_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int) SMEM_MAX);
        });
        if (e != cudaSuccess) return e;
    }
    shard_select_kernel<<<(batch + warps - 1) / warps, 32 * warps, smem, st>>>(
        d, items, n_shards, batch, cand, cand_stride, blo, bhi, sel_out, sel_ws, nsel_ws, status);
    return cudaGetLastError();
}

cudaError_t launch_merge_states(const DevDesc & d, cudaStream_t st, int n_parts, int batch, const float * states,
                                float * out, const uint32_t * flags, const uint32_t * epoch, uint32_t * status) {
    if (flags && (!epoch || !status || n_parts > HEAD_DIM)) return cudaErrorInvalidValue;
    merge_states_kernel<<<dim3(batch, 16), HEAD_DIM, 0, st>>>(d, n_parts, batch, states, out, flags, epoch, status);
    return cudaGetLastError();
}

}  // namespace qsa
