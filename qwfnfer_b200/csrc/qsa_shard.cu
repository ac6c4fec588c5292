// qsa_shard.cu -- the exchange steps of KV-sequence-sharded decode.
//
// The reference runs on one device (README.md:215); sharding the KV sequence axis across GPUs is
// this library's addition for very long contexts.  Rank g owns blocks [blo, bhi) of every layer.
// One step: every rank scores its blocks and keeps its local best (score_select_kernel in sharded
// mode); the candidates of all ranks are all-gathered by the caller; shard_select_kernel forms
// the exact global selection on every rank (every global winner is in its owner's local best);
// each rank attends its own selected blocks into an unnormalised state (attn_kernel, state mode);
// the states are all-gathered and merge_states_kernel combines them by log-sum-exp in rank order.
#include "qsa_kernels.cuh"

namespace qsa {

constexpr int SHARD_SEL_THREADS = 1024;

// Forced blocks of the query at q (the same rule as the selection kernel).
__device__ __forceinline__ void shard_forced_range(const DevDesc & d, int q, int & f_lo, int & f_hi) {
    const int bq = q / d.ratio;
    if (d.window > 0) { f_lo = max(0, bq - d.n_force + 1); f_hi = bq; }
    else if ((q + 1) % d.ratio != 0) { f_lo = bq; f_hi = bq; }
    else { f_lo = 1; f_hi = 0; }
}

// Bitonic sort of n (a power of two) 64-bit keys in shared memory, descending.
__device__ void bitonic_desc(unsigned long long * key, int n) {
    for (int k = 2; k <= n; k <<= 1) {
        for (int j = k >> 1; j > 0; j >>= 1) {
            for (int i = threadIdx.x; i < n; i += blockDim.x) {
                const int ixj = i ^ j;
                if (ixj > i) {
                    const unsigned long long a = key[i], b = key[ixj];
                    const bool desc = (i & k) == 0;
                    if (desc ? (a < b) : (a > b)) { key[i] = b; key[ixj] = a; }
                }
            }
            __syncthreads();
        }
    }
}

// One CTA per query.  Candidates: int32 [n_shards][2][batch][kb], per shard the block ids
// (-1 = none), then the f32 scores' bits.  Writes the global selection (ascending, -1 padded) to
// sel_out (optional) and this rank's blocks [blo, bhi) of it to the workspace list the attention
// kernel reads.
__global__ void __launch_bounds__(SHARD_SEL_THREADS) shard_select_kernel(DevDesc d,
        const qsa_decode_item * __restrict__ items, int n_shards, int batch,
        const int * __restrict__ cand, int blo, int bhi,
        int * __restrict__ sel_out, int * __restrict__ sel_ws, int * __restrict__ nsel_ws,
        uint32_t * __restrict__ status) {
    extern __shared__ __align__(16) unsigned long long keys[];     // [npow2]
    __shared__ int chosen[MAX_KB];
    __shared__ int n_chosen;
    const int t = blockIdx.x;
    const int q = items[t].n_past;
    const int kb = d.kb;
    if (q < 0 || q >= d.n_ctx) {
        if (threadIdx.x == 0) { set_status(status, DEV_BAD_POS); nsel_ws[t] = 0; }
        for (int i = threadIdx.x; i < kb; i += blockDim.x) {
            sel_ws[(size_t) t * kb + i] = -1;
            if (sel_out) sel_out[(size_t) t * kb + i] = -1;
        }
        return;
    }
    int f_lo, f_hi;
    shard_forced_range(d, q, f_lo, f_hi);
    const int n_forced = f_hi >= f_lo ? f_hi - f_lo + 1 : 0;
    const int want = max(0, kb - n_forced);
    const int n = n_shards * kb;
    int np2 = 1;
    while (np2 < n) np2 <<= 1;
    const int n_vis = (q + 1) / d.ratio;
    // key = score bits (non-negative scores order as unsigned) : complement of the block id, so a
    // descending sort orders by score, then lower block first; empty slots are 0 (last).  A
    // candidate that no shard could have sent (not visible, forced, or a negative score) is
    // dropped and flagged.
    for (int i = threadIdx.x; i < np2; i += blockDim.x) {
        unsigned long long k = 0;
        if (i < n) {
            const int sh = i / kb, j = i % kb;
            const size_t o = ((size_t) sh * 2 * batch + t) * kb + j;
            const int b = cand[o];
            if (b >= 0) {
                const uint32_t sbits = (uint32_t) cand[o + (size_t) batch * kb];
                if (b >= n_vis || (b >= f_lo && b <= f_hi) || (sbits >> 31) != 0u || sbits > 0x7f800000u)
                    set_status(status, DEV_BAD_SEL);
                else
                    k = ((unsigned long long) sbits << 32) | (0xffffffffu - (unsigned) b);
            }
        }
        keys[i] = k;
    }
    if (threadIdx.x == 0) n_chosen = 0;
    __syncthreads();
    bitonic_desc(keys, np2);
    // the best `want` candidates plus the forced blocks
    for (int i = threadIdx.x; i < want; i += blockDim.x) {
        const unsigned long long k = keys[i];
        if (k != 0ull) chosen[atomicAdd(&n_chosen, 1)] = (int) (0xffffffffu - (unsigned) (k & 0xffffffffull));
    }
    for (int b = f_lo + (int) threadIdx.x; b <= f_hi; b += blockDim.x) chosen[atomicAdd(&n_chosen, 1)] = b;
    __syncthreads();
    // ascending order: rank each by counting the smaller ones (equal ids, which only a caller
    // that sent one block from two shards produces, by their slot)
    const int m = n_chosen;
    __shared__ int asc[MAX_KB];
    for (int i = threadIdx.x; i < m; i += blockDim.x) {
        const int b = chosen[i];
        int rank = 0;
        for (int j = 0; j < m; j++) rank += chosen[j] < b || (chosen[j] == b && j < i);
        asc[rank] = b;
    }
    __syncthreads();
    if (sel_out)
        for (int i = threadIdx.x; i < kb; i += blockDim.x) sel_out[(size_t) t * kb + i] = i < m ? asc[i] : -1;
    if (threadIdx.x == 0) {                       // this rank's blocks, ascending, for the attention
        int c = 0;
        for (int i = 0; i < m; i++)
            if (asc[i] >= blo && asc[i] < bhi) sel_ws[(size_t) t * kb + c++] = asc[i];
        nsel_ws[t] = c;
    }
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
        int batch, const int * cand, int blo, int bhi, int * sel_out, int * sel_ws, int * nsel_ws, uint32_t * status) {
    int np2 = 1;
    while (np2 < n_shards * d.kb) np2 <<= 1;
    const size_t smem = (size_t) np2 * 8;
    if (smem > 200 * 1024) return cudaErrorInvalidValue;
    cudaError_t e = cudaFuncSetAttribute(shard_select_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
    if (e != cudaSuccess) return e;
    shard_select_kernel<<<batch, SHARD_SEL_THREADS, smem, st>>>(d, items, n_shards, batch, cand, blo, bhi, sel_out,
                                                                sel_ws, nsel_ws, status);
    return cudaGetLastError();
}

cudaError_t launch_merge_states(const DevDesc & d, cudaStream_t st, int n_parts, int batch, const float * states,
                                float * out) {
    merge_states_kernel<<<dim3(batch, 16), HEAD_DIM, 0, st>>>(d, n_parts, batch, states, out);
    return cudaGetLastError();
}

}  // namespace qsa
