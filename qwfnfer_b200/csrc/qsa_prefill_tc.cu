// qsa_prefill_tc.cu -- prefill indexer scores on the 5th-generation tensor cores, and a
// warp-per-query top-k over precomputed scores.
//
// Reference: the prefill scores of graph_builder::qsa_top_k (src/qwfn_graph.cpp:277-293): one
// [n_blocks x (idx_n_head*T)] product of the pooled keys with the indexer queries, relu per head,
// sum over heads; then ggml_top_k per query (:295-306) over score + bias, whose rule
// (src/qwfn_engine.cpp:936-950) the selection below applies directly.
//
// idx_scores_tc_kernel: CTA tile = 128 (query, head) rows x 256 blocks x 128 dims.  The indexer
// queries (f32, rounded to f16 as the reference's vec_dot conversion does) and the F16 pooled keys
// are written to shared memory in the 128-byte-swizzled K-major layout, one elected thread issues
// 8 tcgen05.mma (kind::f16, M=128, N=256, K=16) into a 256-column TMEM accumulator and commits to an
// mbarrier; 8 warps read the accumulator back (tcgen05.ld 32x32b), apply relu, sum the heads of a
// query across lanes and store f32 scores.  Products of f16 values are exact; the sums are f32
// (the reference sums in f32 as well), so scores can differ from an exactly rounded sum by a few
// ulp and the selection only at near-ties.
//
// select_scores_warp_kernel: one warp per query.  Keys are the bit patterns of the non-negative
// scores of the candidate blocks (visible and not forced); a radix select with 8-bit digits from
// the top finds the cut (coalesced passes over the row), then the warp emits the kept blocks 32 at
// a time in ascending order with ballots (equal keys at the cut kept by lower block index), then
// the forced blocks.
#include "qsa_kernels.cuh"
#include "qsa_tc.cuh"

namespace qsa {

constexpr int TC_M = 128;                 // rows (query, head) per CTA
constexpr int TC_N = 256;                 // blocks per CTA
constexpr int TC_K = 128;                 // indexer dims (MAX_IDX_DIM)
constexpr int TC_THREADS = 256;
constexpr int TC_A_BYTES = TC_M * TC_K * 2;      // 32 KB
constexpr int TC_B_BYTES = TC_N * TC_K * 2;      // 64 KB
constexpr int TC_SMEM = TC_A_BYTES + TC_B_BYTES + 1024;   // + alignment slack for the 1024-byte swizzle atoms

// Instruction descriptor, kind::f16: D f32, A and B f16, both K-major, N = 256, M = 128.
constexpr uint32_t TC_IDESC = umma_idesc_f16(TC_M, TC_N);

__global__ void __launch_bounds__(TC_THREADS) idx_scores_tc_kernel(DevDesc d, const float * __restrict__ q_idx,
        int n_rows, const uint16_t * __restrict__ pool, int n_blocks, float * __restrict__ scores, int scores_stride,
        uint32_t * __restrict__ status) {
    extern __shared__ __align__(1024) unsigned char tc_smem_raw[];
    __shared__ uint64_t mma_bar;
    __shared__ uint32_t tmem_slot;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int row0 = blockIdx.x * TC_M, blk0 = blockIdx.y * TC_N;
    // 1024-byte aligned operand tiles
    const uint32_t raw = smem_u32(tc_smem_raw);
    const uint32_t base = (raw + 1023u) & ~1023u;
    unsigned char * sA = tc_smem_raw + (base - raw);
    unsigned char * sB = sA + TC_A_BYTES;

    if (warp == 0) tmem_alloc_warp(&tmem_slot, TC_N);   // TMEM accumulator: 128 lanes x 256 f32 columns
    if (tid == 0) {
        mbar_init(&mma_bar, 1);
        fence_mbar_init();
    }
    // A: (query, head) rows of the indexer query, f32 -> f16 (RNE), 16-byte chunks
    for (int i = tid; i < TC_M * (TC_K / 8); i += TC_THREADS) {
        const int r = i >> 4, c = i & 15;
        uint4 v = make_uint4(0, 0, 0, 0);
        if (row0 + r < n_rows) {
            const float4 * src = reinterpret_cast<const float4 *>(q_idx + (size_t) (row0 + r) * TC_K + 8 * c);
            const float4 a = __ldg(src), b = __ldg(src + 1);
            v.x = pack_f16x2(a.x, a.y); v.y = pack_f16x2(a.z, a.w);
            v.z = pack_f16x2(b.x, b.y); v.w = pack_f16x2(b.z, b.w);
        }
        *reinterpret_cast<uint4 *>(sA + sw128_off(TC_M, r, 8 * c)) = v;
    }
    // B: pooled keys of blocks blk0 .. blk0+255 (already F16)
    for (int i = tid; i < TC_N * (TC_K / 8); i += TC_THREADS) {
        const int r = i >> 4, c = i & 15;
        uint4 v = make_uint4(0, 0, 0, 0);
        if (blk0 + r < n_blocks) v = __ldg(reinterpret_cast<const uint4 *>(pool + (size_t) (blk0 + r) * TC_K + 8 * c));
        *reinterpret_cast<uint4 *>(sB + sw128_off(TC_N, r, 8 * c)) = v;
    }
    fence_async_smem();                       // operands visible to the tensor core
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tmem_slot;
    if (tid == 0) {
        #pragma unroll
        for (int k = 0; k < TC_K / 16; k++) {
            // k-step k: columns 16k .. 16k+15 = atom k/4, byte offset 32 (k%4) inside the swizzled rows
            const uint64_t da = umma_desc_sw128(base + (uint32_t) ((k >> 2) * TC_M * 128 + (k & 3) * 32));
            const uint64_t db = umma_desc_sw128(base + TC_A_BYTES + (uint32_t) ((k >> 2) * TC_N * 128 + (k & 3) * 32));
            umma_f16(tmem, da, db, TC_IDESC, k > 0);
        }
        umma_commit(&mma_bar);
    }
    const bool ok = mbar_wait_bounded(&mma_bar, 0, status);
    tc_fence_after();
    // Epilogue: warp w reads TMEM lanes 32 (w % 4) .. +31 (its rows), columns 128 (w / 4) .. +127.
    const int H = d.idx_n_head;
    const int sub = warp & 3, chalf = warp >> 2;
    const int r = sub * 32 + lane;                     // tile row = TMEM lane
    const int grow = row0 + r;                         // global (query, head) row
    const int t = grow / H, h = grow - t * H;
    #pragma unroll 1
    for (int c0 = chalf * 128; c0 < chalf * 128 + 128; c0 += 32) {
        uint32_t v[32];
        tmem_ld32(tmem + ((uint32_t) (sub * 32) << 16) + (uint32_t) c0, v);
        tmem_ld_wait();
        float s[32];
        #pragma unroll
        for (int j = 0; j < 32; j++) {
            const float x = __uint_as_float(v[j]);
            s[j] = x > 0.0f ? x : 0.0f;                // relu per head
        }
        // sum over the heads of a query: its H rows are consecutive lanes (H divides 32)
        for (int off = 1; off < H; off <<= 1)
            #pragma unroll
            for (int j = 0; j < 32; j++) s[j] += __shfl_xor_sync(0xffffffffu, s[j], off);
        if (ok && h == 0 && grow < n_rows) {
            float * dst = scores + (size_t) t * scores_stride + blk0 + c0;
            const int nvalid = min(32, n_blocks - (blk0 + c0));
            if (nvalid == 32) {
                #pragma unroll
                for (int j = 0; j < 32; j += 4)
                    *reinterpret_cast<float4 *>(dst + j) = make_float4(s[j], s[j + 1], s[j + 2], s[j + 3]);
            } else {
                for (int j = 0; j < nvalid; j++) dst[j] = s[j];
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc_warp(tmem, TC_N);
    }
}

// ---------------------------------------------------------------------------------------------
constexpr int SELW_WARPS = 8;             // queries per CTA

// One warp per query t (prefill: position n_past0 + t); scores row t of `scores` (stride
// scores_stride) holds the candidates' head-summed relu scores.
__global__ void __launch_bounds__(32 * SELW_WARPS) select_scores_warp_kernel(DevDesc d, int n_past0, int n_q,
        const float * __restrict__ scores, int scores_stride, int * __restrict__ sel_ws, int * __restrict__ nsel_ws,
        int * __restrict__ sel_out, uint32_t * __restrict__ status) {
    __shared__ unsigned hist[SELW_WARPS][256];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int t = blockIdx.x * SELW_WARPS + warp;
    if (t >= n_q) return;
    const int q = n_past0 + t;
    int * sel = sel_ws + (size_t) t * d.kb;
    int * so = sel_out ? sel_out + (size_t) t * d.kb : nullptr;
    if (q < 0 || q >= d.n_ctx || (q + 1) / d.ratio > scores_stride) {
        if (lane == 0) { set_status(status, DEV_BAD_POS); nsel_ws[t] = 0; }
        for (int i = lane; i < d.kb; i += 32) { sel[i] = -1; if (so) so[i] = -1; }
        return;
    }
    const int n_vis = (q + 1) / d.ratio;
    const int bq = q / d.ratio;
    int f_lo, f_hi;
    if (d.window > 0) { f_lo = max(0, bq - d.n_force + 1); f_hi = bq; }
    else if ((q + 1) % d.ratio != 0) { f_lo = bq; f_hi = bq; }
    else { f_lo = 1; f_hi = 0; }
    const int n_forced = f_hi >= f_lo ? f_hi - f_lo + 1 : 0;
    const int cand_hi = n_forced ? min(n_vis, f_lo) : n_vis;   // candidates: [0, cand_hi)
    const int want = max(0, d.kb - n_forced);
    const float * sc = scores + (size_t) t * scores_stride;
    // lane l visits candidates l, l + 32, ...: every warp load reads 128 contiguous bytes, and the
    // row (a few KB) stays in L1 across the passes
    uint32_t prefix = 0, pmask = 0;
    int remaining = want;
    const bool take_none = want == 0;
    const bool take_all = !take_none && cand_hi <= want;
    unsigned * hw = hist[warp];
    if (!take_all && !take_none) {
        for (int shift = 24; shift >= 0; shift -= 8) {
            for (int i = lane; i < 256; i += 32) hw[i] = 0;
            __syncwarp();
            int b = lane;
            for (; b + 96 < cand_hi; b += 128) {
                uint32_t k4[4];
                #pragma unroll
                for (int u = 0; u < 4; u++) k4[u] = __float_as_uint(__ldg(sc + b + 32 * u));
                #pragma unroll
                for (int u = 0; u < 4; u++)
                    if ((k4[u] & pmask) == prefix) atomicAdd(&hw[(k4[u] >> shift) & 255u], 1u);
            }
            for (; b < cand_hi; b += 32) {
                const uint32_t key = __float_as_uint(__ldg(sc + b));
                if ((key & pmask) == prefix) atomicAdd(&hw[(key >> shift) & 255u], 1u);
            }
            __syncwarp();
            // lane owns bins 255-8*lane .. 248-8*lane (from the top); suffix counts across lanes
            int own = 0;
            #pragma unroll
            for (int k = 0; k < 8; k++) own += (int) hw[255 - 8 * lane - k];
            int incl = own;
            #pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int y = __shfl_up_sync(0xffffffffu, incl, o);
                if (lane >= o) incl += y;
            }
            const int above = incl - own;
            const unsigned hit = __ballot_sync(0xffffffffu, above < remaining && incl >= remaining);
            const int src = __ffs(hit) - 1;
            int bin = 0, cut_rem = 0;
            if (lane == src) {
                int cum = above;
                int k = 0;
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
    // emission in ascending block order, 32 blocks at a time: keys above the cut are kept, keys
    // equal to it (all 32 bits) by lower block index, `remaining` of them
    const unsigned lt = (1u << lane) - 1u;
    int n_cand_taken = 0, eq_seen = 0;
    if (!take_none) {
        for (int b0 = 0; b0 < cand_hi; b0 += 32) {
            const int b = b0 + lane;
            bool above = false, eq = false;
            if (b < cand_hi) {
                if (take_all) {
                    above = true;
                } else {
                    const uint32_t key = __float_as_uint(__ldg(sc + b));
                    above = key > prefix;
                    eq = key == prefix;
                }
            }
            const unsigned eqb = __ballot_sync(0xffffffffu, eq);
            const bool tk = above || (eq && eq_seen + __popc(eqb & lt) < remaining);
            const unsigned tb = __ballot_sync(0xffffffffu, tk);
            const int pos = n_cand_taken + __popc(tb & lt);
            if (tk && pos < d.kb) { sel[pos] = b; if (so) so[pos] = b; }
            n_cand_taken += __popc(tb);
            eq_seen += __popc(eqb);
        }
    }
    // forced blocks follow (they are above every candidate)
    for (int i = lane; i < n_forced; i += 32) {
        const int p = n_cand_taken + i;
        if (p < d.kb) { sel[p] = f_lo + i; if (so) so[p] = f_lo + i; }
    }
    const int n = min(d.kb, n_cand_taken + n_forced);
    for (int i = n + lane; i < d.kb; i += 32) { sel[i] = -1; if (so) so[i] = -1; }
    if (lane == 0) nsel_ws[t] = n;
}

cudaError_t launch_prefill_scores_tc(const DevDesc & d, cudaStream_t st, const float * q_idx, int T,
                                     const uint16_t * pool, int n_blocks, float * scores, int scores_stride,
                                     uint32_t * status) {
    static std::atomic<uint64_t> attr{0};
    const cudaError_t e = once_per_device(attr, [] {
        return cudaFuncSetAttribute(idx_scores_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, TC_SMEM);
    });
    if (e != cudaSuccess) return e;
    const int n_rows = T * d.idx_n_head;
    const dim3 grid((unsigned) ((n_rows + TC_M - 1) / TC_M), (unsigned) ((n_blocks + TC_N - 1) / TC_N));
    if (n_blocks <= 0) return cudaSuccess;
    idx_scores_tc_kernel<<<grid, TC_THREADS, TC_SMEM, st>>>(d, q_idx, n_rows, pool, n_blocks, scores, scores_stride,
                                                            status);
    return cudaGetLastError();
}

cudaError_t launch_select_scores_warp(const DevDesc & d, cudaStream_t st, int n_past0, int T, const float * scores,
                                      int scores_stride, int * sel_ws, int * nsel_ws, int * sel_out, uint32_t * status) {
    select_scores_warp_kernel<<<(T + SELW_WARPS - 1) / SELW_WARPS, 32 * SELW_WARPS, 0, st>>>(
        d, n_past0, T, scores, scores_stride, sel_ws, nsel_ws, sel_out, status);
    return cudaGetLastError();
}

}  // namespace qsa
