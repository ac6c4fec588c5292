// qsa_prefill_attn.cu -- KV-stationary sparse attention of a prefill chunk on the 5th-generation
// tensor cores.
//
// Reference: the prefill attention of graph_builder::sparse_attn (src/qwfn_graph.cpp:362-403):
// ggml_flash_attn_ext of the chunk's queries over the cache with a mask that keeps, per query, the
// cells of its selected blocks that are not in its future.
//
// Every query of a chunk selects its own blocks, so a query-major pass re-reads each block for
// every query that selected it (about 200 times per block in an 8192-token chunk).  Here the work
// is grouped by block instead:
//   1. prefill_bucket_*: the (query, slot) pairs of the chunk's selections are bucketed by block
//      (counting sort: counts, one scan, a fill that also records each pair's bucket position,
//      its "entry"); prefill_q16_kernel converts Q to f16 rows;
//   2. prefill_attn_kv_kernel, CTA = (block, KV head): the block's raw K and V rows of that head
//      come in by TMA and are dequantised once into shared memory (f16 of d x q, the rounding of
//      the reference's decode gather); then the CTA walks its entries 16 at a time (16 queries x 8
//      query heads = 128 rows) in a warp-specialised pipeline:
//        warp 8      TMA loads of the queries' Q rows (one 4 KB box per query) into one of two
//                    Q stages
//        warp 9      one thread issues S = Q K^T (16 tcgen05.mma, M=128, N=64 cells, K=16) into one
//                    of two TMEM S buffers, and O = P V (4 tcgen05.mma, M=128, N=256, K=16) into
//                    TMEM, each as soon as its inputs are ready (non-blocking barrier tests); the
//                    S commit also releases the Q stage
//        warps 0-3   thread = row = TMEM lane: S from TMEM, mask of the cells past the query,
//                    P = 2^(s - m) (f16) -> shared memory, row maximum and sum
//        warps 4-7   thread = row: O / l from TMEM into registers (f16), release O, then each
//                    warp writes its 32 rows through a 2 KB slice (8 rows x 64 bytes per store
//                    instruction), and (m, l) of each row
//      The partials are entry-major, [KV head][entry][8 query heads][256 dims] f16, so a chunk's
//      rows are contiguous;
//   3. prefill_merge_kernel: per query, a warp per head merges its slots' partials (log-sum-exp),
//      finding each slot's row through the entry recorded for it.
// Tensor-core operands use the 128-byte swizzle: Q [16 queries][4 atoms of 64 dims][8 rows] (K-major,
// 8-row groups 4 KB apart), K and V [64 cells][256 dims] (K-major for S; V as the MN-major B of
// O = P V), P [128 rows][64 cells] (K-major).
#include "qsa_kernels.cuh"
#include "qsa_tc.cuh"
#include "qsa_tma.cuh"

namespace qsa {

constexpr int PA_THREADS = 320;                    // warps 0-3 softmax, 4-7 epilogue, 8 loads, 9 MMA
constexpr int PA_QC = 16;                          // queries per chunk
constexpr int PA_ROWS = PA_QC * GQA_TILE;          // 128 MMA rows
constexpr int PA_CELLS = 64;                       // cells of a block (ratio 64)
constexpr int PA_SQ = PA_ROWS * HEAD_DIM * 2;      // 64 KB
constexpr int PA_SK = PA_CELLS * HEAD_DIM * 2;     // 32 KB
constexpr int PA_SV = HEAD_DIM * PA_CELLS * 2;     // 32 KB
constexpr int PA_SP = PA_ROWS * PA_CELLS * 2;      // 16 KB
constexpr int PA_SW = 32 * 64;                      // 2 KB per epilogue warp: 32 rows x 64 bytes
constexpr int PA_SMEM = 2 * PA_SQ + PA_SK + PA_SV + PA_SP + 4 * PA_SW + 1024;
constexpr int PA_HEAD_Q8 = HEAD_DIM / QK8_0 * Q8_0_BYTES;   // 272 bytes of one head's q8_0 row
constexpr int PA_QROWS = 8 * HEAD_DIM * 2;         // 4 KB: one query's 8 head rows in a Q stage
constexpr uint32_t PA_TMEM_COLS = 512;             // S buffers: columns 0..63, 64..127; O: 256..511
constexpr uint32_t PA_TMEM_O = 256;
constexpr uint32_t PA_IDESC_S = umma_idesc_f16(PA_ROWS, PA_CELLS);
constexpr uint32_t PA_IDESC_O = umma_idesc_f16(PA_ROWS, HEAD_DIM) | (1u << 16);   // B (V) MN-major
constexpr int PA_SLOT_SHIFT = 10;                  // entry = query << 10 | slot (slot < MAX_KB)
// A Q stage is [query][64-column atom][8 rows][128 bytes] with the 128-byte swizzle inside each
// 1 KB (8 rows x 128 bytes): the MMA reads it as a K-major operand whose 8-row groups are 4 KB
// apart, and one 4-D TMA box moves a query's 4 KB.
// shared-memory descriptor of a 128-byte-swizzled MN-major operand: 64-element MN blocks lbo bytes
// apart, groups of 8 K rows (1 KB atoms) sbo bytes apart
__device__ __forceinline__ uint64_t umma_desc_sw128_mn(uint32_t smem_addr, uint32_t lbo, uint32_t sbo) {
    return (uint64_t) ((smem_addr >> 4) & 0x3FFFu) | ((uint64_t) ((lbo >> 4) & 0x3FFFu) << 16) |
           ((uint64_t) ((sbo >> 4) & 0x3FFFu) << 32) | ((uint64_t) 1 << 46) | ((uint64_t) 2 << 61);
}
// shared-memory descriptor of a 128-byte-swizzled K-major operand whose 8-row groups are sbo bytes apart
__device__ __forceinline__ uint64_t umma_desc_sw128_sbo(uint32_t smem_addr, uint32_t sbo) {
    return (uint64_t) ((smem_addr >> 4) & 0x3FFFu) | ((uint64_t) 1 << 16) | ((uint64_t) ((sbo >> 4) & 0x3FFFu) << 32) |
           ((uint64_t) 1 << 46) | ((uint64_t) 2 << 61);
}

// ------------------------------------------------------------------ bucketing by block
__global__ void prefill_bucket_count_kernel(const DevDesc d, int T, const int * __restrict__ sel,
                                            const int * __restrict__ nsel, int n_blocks, int * __restrict__ cnt) {
    const int64_t i = (int64_t) blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (int64_t) T * d.kb) return;
    const int t = (int) (i / d.kb), j = (int) (i % d.kb);
    if (j >= nsel[t]) return;
    const int b = sel[i];
    if (b >= 0 && b < n_blocks) atomicAdd(&cnt[b], 1);
}

// one CTA: exclusive scan of the counts into offsets[0..n_blocks] and the fill cursors
__global__ void __launch_bounds__(1024) prefill_bucket_scan_kernel(const int * __restrict__ cnt, int n_blocks,
                                                                   int * __restrict__ offsets, int * __restrict__ cursor) {
    __shared__ int wsum[32];
    __shared__ int carry;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    if (tid == 0) carry = 0;
    __syncthreads();
    for (int base = 0; base < n_blocks; base += 1024) {
        const int i = base + tid;
        const int v = i < n_blocks ? cnt[i] : 0;
        int x = v;
        #pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int y = __shfl_up_sync(0xffffffffu, x, o);
            if (lane >= o) x += y;
        }
        if (lane == 31) wsum[warp] = x;
        __syncthreads();
        if (warp == 0) {
            int w = wsum[lane], y = w;
            #pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int z = __shfl_up_sync(0xffffffffu, y, o);
                if (lane >= o) y += z;
            }
            wsum[lane] = y - w;
        }
        __syncthreads();
        const int excl = carry + wsum[warp] + x - v;
        if (i < n_blocks) { offsets[i] = excl; cursor[i] = excl; }
        __syncthreads();
        if (tid == 1023) carry = excl + v;
        __syncthreads();
    }
    if (tid == 0) offsets[n_blocks] = carry;
}

// entries[pos] = query << 10 | slot, and entry_of[query * kb + slot] = pos (-1 for no block)
__global__ void prefill_bucket_fill_kernel(const DevDesc d, int T, const int * __restrict__ sel,
                                           const int * __restrict__ nsel, int n_blocks, int * __restrict__ cursor,
                                           uint32_t * __restrict__ entries, int * __restrict__ entry_of) {
    const int64_t i = (int64_t) blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (int64_t) T * d.kb) return;
    const int t = (int) (i / d.kb), j = (int) (i % d.kb);
    const int b = j < nsel[t] ? sel[i] : -1;
    if (b < 0 || b >= n_blocks) {
        entry_of[i] = -1;
        return;
    }
    const int pos = atomicAdd(&cursor[b], 1);
    entries[pos] = ((uint32_t) t << PA_SLOT_SHIFT) | (uint32_t) j;
    entry_of[i] = pos;
}

// Q (bf16 or f32, [T][n_head][256]) -> f16 rows [T * n_head][256], 8 values per thread
__global__ void prefill_q16_kernel(const void * __restrict__ q, int q_type, int64_t n8, uint4 * __restrict__ q16) {
    const int64_t i = (int64_t) blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n8) return;
    float f[8];
    if (q_type == QSA_TYPE_BF16) {
        const uint4 x = reinterpret_cast<const uint4 *>(q)[i];
        const uint32_t xx[4] = {x.x, x.y, x.z, x.w};
        #pragma unroll
        for (int k = 0; k < 4; k++) { f[2 * k] = __uint_as_float(xx[k] << 16); f[2 * k + 1] = __uint_as_float(xx[k] & 0xffff0000u); }
    } else {
        const float4 x0 = reinterpret_cast<const float4 *>(q)[2 * i], x1 = reinterpret_cast<const float4 *>(q)[2 * i + 1];
        f[0] = x0.x; f[1] = x0.y; f[2] = x0.z; f[3] = x0.w; f[4] = x1.x; f[5] = x1.y; f[6] = x1.z; f[7] = x1.w;
    }
    q16[i] = make_uint4(pack_f16x2(f[0], f[1]), pack_f16x2(f[2], f[3]), pack_f16x2(f[4], f[5]), pack_f16x2(f[6], f[7]));
}

// ------------------------------------------------------------------ attention per (block, KV head)
// Bytes 0 and 2 of t (int8) times the f16 scale, as f16x2: the bytes become exact f16 integers and
// the f16 multiply rounds d x q once, as the reference's f16(f32(d) * q) does (that f32 product is
// exact).
__device__ __forceinline__ uint32_t i8x2_scaled(uint32_t t, __half2 d) {
    const uint32_t x = i8x2_even_to_f16x2(t);
    const __half2 r = __hmul2(*reinterpret_cast<const __half2 *>(&x), d);
    return *reinterpret_cast<const uint32_t *>(&r);
}

struct PaBarriers {
    uint64_t kv_full;                 // raw q8_0 rows of the block copied in (bulk-copy bytes)
    uint64_t q_full[2], q_empty[2];   // Q stage loaded (TMA bytes) / read by its S MMAs (commit)
    uint64_t s_full[2], s_empty[2];   // S buffer written (commit) / read by the 128 softmax threads
    uint64_t p_full, p_empty;         // sP written by the softmax threads / read by the O MMAs (commit)
    uint64_t o_full, o_empty;         // O in TMEM (commit) / read by the 128 epilogue threads
    uint64_t meta_full[2];            // row statistics of a chunk written by the softmax threads
    uint64_t mma_done;                // the MMA thread's last commit before TMEM is released
};

__global__ void __launch_bounds__(PA_THREADS, 1) prefill_attn_kv_kernel(
        const __grid_constant__ CUtensorMap q_map, const __grid_constant__ CUtensorMap k_map,
        const __grid_constant__ CUtensorMap v_map, DevDesc d, int n_past0, int n_kv, int slots,
        const uint32_t * __restrict__ entries, const int * __restrict__ offsets, __half * __restrict__ part_o,
        float * __restrict__ part_ml, uint32_t * __restrict__ status) {
    extern __shared__ __align__(1024) unsigned char pa_smem_raw[];
    __shared__ PaBarriers bars;
    __shared__ uint32_t tmem_slot;
    __shared__ float row_m[2][PA_ROWS], row_l[2][PA_ROWS];
    const int b = blockIdx.x, g = blockIdx.y;
    const int e0 = offsets[b], e1 = offsets[b + 1];
    if (e0 >= e1) return;                                   // no query selected this block
    const int n_chunks = (e1 - e0 + PA_QC - 1) / PA_QC;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const uint32_t raw = smem_u32(pa_smem_raw);
    const uint32_t base = (raw + 1023u) & ~1023u;
    unsigned char * sQ0 = pa_smem_raw + (base - raw);       // two Q stages; a stage also holds the
    unsigned char * sK = sQ0 + 2 * PA_SQ;                   // O rows of its chunk for the TMA stores
    unsigned char * sV = sK + PA_SK;                        // V [64 cells][256 dims], like K
    unsigned char * sP = sV + PA_SV;
    unsigned char * sW = sP + PA_SP;                        // the epilogue warps' row pieces
    const uint32_t aQ0 = base, aK = base + 2 * PA_SQ, aV = aK + PA_SK, aP = aV + PA_SV;
    // the raw q8_0 rows (head g: 272 bytes of a 544-byte row) land in Q stage 1 before chunk 1 does
    unsigned char * rawK = sQ0 + PA_SQ;
    unsigned char * rawV = rawK + PA_CELLS * PA_HEAD_Q8;
    const int n_valid = min(PA_CELLS, n_kv - b * PA_CELLS);
    const bool kv_f16 = d.type_k == QSA_TYPE_F16;

    if (warp == 0) tmem_alloc_warp(&tmem_slot, PA_TMEM_COLS);
    if (tid == 32) {
        mbar_init(&bars.kv_full, 1);
        for (int k = 0; k < 2; k++) {
            mbar_init(&bars.q_full[k], 1);
            mbar_init(&bars.q_empty[k], 1);
            mbar_init(&bars.s_full[k], 1);
            mbar_init(&bars.s_empty[k], PA_ROWS);
            mbar_init(&bars.meta_full[k], PA_ROWS);
        }
        mbar_init(&bars.p_full, PA_ROWS);
        mbar_init(&bars.p_empty, 1);
        mbar_init(&bars.o_full, 1);
        mbar_init(&bars.o_empty, PA_ROWS);
        mbar_init(&bars.mma_done, 1);
        fence_mbar_init();
    }
    __syncthreads();
    auto chunk_entry = [&](int i, int k) -> uint32_t {     // entry k of chunk i, or ~0u past its end
        const int c = e0 + i * PA_QC + k;
        return k < PA_QC && c < e1 ? entries[c] : ~0u;
    };
    // Q rows of chunk i into stage i % 2 (the whole loader warp; lane k holds entry k of the chunk)
    auto load_q = [&](int i, uint32_t e) {
        const int s = i & 1, nq = min(PA_QC, e1 - (e0 + i * PA_QC));
        if (lane == 0) mbar_arrive_expect_tx(&bars.q_full[s], (uint32_t) (nq * PA_QROWS));
        __syncwarp();
        if (lane < nq)          // query t's rows of KV head g: 8-row group t * n_head_kv + g of Q
            tma_load_4d(aQ0 + s * PA_SQ + lane * PA_QROWS, &q_map, (int) (e >> PA_SLOT_SHIFT) * d.n_head_kv + g,
                        &bars.q_full[s]);
    };
    if (warp == 8) {
        if (lane == 0) {
            if (kv_f16) {
                // f16 caches: head g's K and V tiles straight into the swizzled [cell][dim] layout
                // (atoms 4g..4g+3 of the rows; cells past n_kv are zeroed below)
                mbar_arrive_expect_tx(&bars.kv_full, (uint32_t) (PA_SK + PA_SV));
                tma_load_3d(aK, &k_map, 0, b * PA_CELLS, 4 * g, &bars.kv_full);
                tma_load_3d(aV, &v_map, 0, b * PA_CELLS, 4 * g, &bars.kv_full);
            } else {
                // q8_0: the block's raw rows of head g, one box of 64 rows x 272 bytes each (the bytes
                // of cells past n_kv are fetched too, and ignored)
                mbar_arrive_expect_tx(&bars.kv_full, (uint32_t) (2 * PA_CELLS * PA_HEAD_Q8));
                tma_load_2d(smem_u32(rawK), &k_map, g * (PA_HEAD_Q8 / 2), b * PA_CELLS, &bars.kv_full);
                tma_load_2d(smem_u32(rawV), &v_map, g * (PA_HEAD_Q8 / 2), b * PA_CELLS, &bars.kv_full);
            }
        }
        load_q(0, chunk_entry(0, lane));
    }
    mbar_wait_bounded(&bars.kv_full, 0u, status);

    // ---- K and V -> f16 (d x q), both as [cell][dim] (K-major for S = Q K^T, MN-major for O = P V);
    // cells at or past n_kv are zero (their bytes may decode to Inf or NaN, and a masked P of 0
    // times a NaN is NaN in the MMA)
    if (kv_f16) {
        for (int i = tid; i < 2 * (PA_CELLS - n_valid) * (HEAD_DIM / 8); i += PA_THREADS) {
            const int per = (PA_CELLS - n_valid) * (HEAD_DIM / 8);
            const int kv = i >= per, j = i - kv * per, cell = n_valid + (j >> 5), d8 = j & 31;
            *reinterpret_cast<uint4 *>((kv ? sV : sK) + sw128_off(PA_CELLS, cell, d8 * 8)) = make_uint4(0, 0, 0, 0);
        }
    } else
    for (int i = tid; i < 2 * PA_CELLS * (HEAD_DIM / 8); i += PA_THREADS) {   // (K or V, cell, 8-dim group)
        const int kv = i >> 11, cell = (i >> 5) & (PA_CELLS - 1), d8 = i & 31;
        uint4 w = make_uint4(0, 0, 0, 0);
        if (cell < n_valid) {
            const uint8_t * blk = (kv ? rawV : rawK) + cell * PA_HEAD_Q8 + (d8 >> 2) * Q8_0_BYTES;
            const __half2 sc = __half2half2(__ushort_as_half(*reinterpret_cast<const uint16_t *>(blk)));
            const uint32_t lo = lds_u32_a2(blk + 2 + (d8 & 3) * 8), hi = lds_u32_a2(blk + 6 + (d8 & 3) * 8);
            w.x = i8x2_scaled(__byte_perm(lo, 0u, 0x0100), sc);
            w.y = i8x2_scaled(__byte_perm(lo, 0u, 0x0302), sc);
            w.z = i8x2_scaled(__byte_perm(hi, 0u, 0x0100), sc);
            w.w = i8x2_scaled(__byte_perm(hi, 0u, 0x0302), sc);
        }
        *reinterpret_cast<uint4 *>((kv ? sV : sK) + sw128_off(PA_CELLS, cell, d8 * 8)) = w;
    }
    fence_async_smem();                                     // K and V tiles visible to the tensor core,
    tc_fence_before();                                      // and stage 1 free for the TMA
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tmem_slot;

    if (warp == 8) {
        // ---------------------------------------------------------------- Q loads
        int i = 1;
        for (; i < n_chunks; i++) {
            const uint32_t e = chunk_entry(i, lane);
            // stage i % 2 is free once the S MMAs of chunk i-2 are done
            int ok = 1;
            if (i >= 2 && lane == 0) ok = mbar_poll_bounded(&bars.q_empty[i & 1], (uint32_t) (((i - 2) >> 1) & 1), status);
            if (!__shfl_sync(0xffffffffu, ok, 0)) break;
            load_q(i, e);
        }
        // every issued load has landed before the CTA can leave
        mbar_wait_bounded(&bars.q_full[(i - 1) & 1], (uint32_t) (((i - 1) >> 1) & 1), status);
    } else if (warp == 9) {
        // ---------------------------------------------------------------- MMA issue (one thread)
        // S of chunk ns (Q loaded, its S buffer read out) and O of chunk no (P written, the previous
        // O read out) are issued as soon as they are ready, in whichever order that happens
        if (lane == 0) {
            int ns = 0, no = 0;
            uint64_t t_last = global_timer_ns();
            while (no < n_chunks) {
                bool progress = false;
                if (ns < n_chunks && ns <= no + 2) {
                    const int s = ns & 1;
                    if (mbar_test(&bars.q_full[s], (uint32_t) ((ns >> 1) & 1)) &&
                        (ns < 2 || mbar_test(&bars.s_empty[s], (uint32_t) (((ns - 2) >> 1) & 1)))) {
                        tc_fence_after();
                        const uint32_t aQ = aQ0 + s * PA_SQ;
                        #pragma unroll
                        for (int kk = 0; kk < HEAD_DIM / 16; kk++)
                            umma_f16(tmem + (uint32_t) (s * PA_CELLS),
                                     umma_desc_sw128_sbo(aQ + (kk >> 2) * 1024 + (kk & 3) * 32, PA_QROWS),
                                     umma_desc_sw128(aK + (kk >> 2) * (PA_CELLS * 128) + (kk & 3) * 32), PA_IDESC_S, kk > 0);
                        umma_commit(&bars.s_full[s]);
                        umma_commit(&bars.q_empty[s]);
                        ns++;
                        progress = true;
                    }
                }
                if (no < ns && mbar_test(&bars.p_full, (uint32_t) (no & 1)) &&
                    (no < 1 || mbar_test(&bars.o_empty, (uint32_t) ((no - 1) & 1)))) {
                    tc_fence_after();
                    #pragma unroll
                    for (int kk = 0; kk < PA_CELLS / 16; kk++)
                        umma_f16(tmem + PA_TMEM_O, umma_desc_sw128(aP + kk * 32),
                                 umma_desc_sw128_mn(aV + kk * 2048, PA_CELLS * 128, 1024), PA_IDESC_O, kk > 0);
                    umma_commit(&bars.o_full);
                    umma_commit(&bars.p_empty);
                    no++;
                    progress = true;
                }
                const uint64_t now = global_timer_ns();
                if (progress) {
                    t_last = now;
                } else if (now - t_last > 2000000000ull) {
                    set_status(status, DEV_TIMEOUT);
                    break;
                }
            }
            umma_commit(&bars.mma_done);                     // every MMA issued above has completed
            mbar_wait_bounded(&bars.mma_done, 0u, status);
        }
        __syncwarp();
    } else if (warp < 4) {
        // ---------------------------------------------------------------- softmax, thread = row
        const int r = tid, qi = r >> 3;
        const uint32_t lane_base = (uint32_t) (warp * 32) << 16;
        for (int i = 0; i < n_chunks; i++) {
            const int buf = i & 1;
            const uint32_t e = chunk_entry(i, qi);
            int lim = -1;                                     // cells 0..lim of the block are visible
            if (e != ~0u) lim = n_past0 + (int) (e >> PA_SLOT_SHIFT) - b * PA_CELLS;
            if (!mbar_wait_bounded(&bars.s_full[buf], (uint32_t) ((i >> 1) & 1), status)) break;
            tc_fence_after();
            uint32_t v[32], u[32];
            tmem_ld32(tmem + lane_base + (uint32_t) (buf * PA_CELLS), v);
            tmem_ld32(tmem + lane_base + (uint32_t) (buf * PA_CELLS + 32), u);
            tmem_ld_wait();
            tc_fence_before();
            mbar_arrive(&bars.s_empty[buf]);
            float s[64];
            float m = -INFINITY;
            #pragma unroll
            for (int c = 0; c < 32; c++) {
                s[c] = c <= lim ? __uint_as_float(v[c]) * d.scale_log2 : -INFINITY;
                s[32 + c] = 32 + c <= lim ? __uint_as_float(u[c]) * d.scale_log2 : -INFINITY;
            }
            #pragma unroll
            for (int c = 0; c < 64; c++) m = fmaxf(m, s[c]);
            const float mu = m == -INFINITY ? 0.0f : m;
            float l = 0.0f;
            uint32_t pk[32];
            #pragma unroll
            for (int c = 0; c < 32; c++) {
                const float p0 = exp2f(s[2 * c] - mu), p1 = exp2f(s[2 * c + 1] - mu);
                l += p0 + p1;
                pk[c] = pack_f16x2(p0, p1);
            }
            // O of chunk i-1 is done: sP is free, and so is this row-statistics buffer (the epilogue
            // of chunk i-2 read it before releasing the O that chunk i-1 was written into)
            if (i >= 1 && !mbar_wait_bounded(&bars.p_empty, (uint32_t) ((i - 1) & 1), status)) break;
            row_m[buf][r] = m;
            row_l[buf][r] = l;
            mbar_arrive(&bars.meta_full[buf]);
            #pragma unroll
            for (int c8 = 0; c8 < 8; c8++)
                *reinterpret_cast<uint4 *>(sP + sw128_off(PA_ROWS, r, c8 * 8)) =
                    make_uint4(pk[4 * c8], pk[4 * c8 + 1], pk[4 * c8 + 2], pk[4 * c8 + 3]);
            fence_async_smem();
            mbar_arrive(&bars.p_full);
        }
    } else {
        // ---------------------------------------------------------------- epilogue, thread = row
        // O / l of the row as f16 into registers, release O, then the warp's 32 rows go out 64 bytes
        // of a row at a time through a 2 KB slice (8 rows x 64 bytes per store instruction)
        const int r = tid - 128, qi = r >> 3, ew = warp - 4;
        const uint32_t lane_base = (uint32_t) (ew * 32) << 16;
        unsigned char * wbuf = sW + ew * PA_SW;
        for (int i = 0; i < n_chunks; i++) {
            const int buf = i & 1;
            const int c0 = e0 + i * PA_QC, nq = min(PA_QC, e1 - c0);
            bool ok = mbar_wait_bounded(&bars.meta_full[buf], (uint32_t) ((i >> 1) & 1), status);
            const float m = row_m[buf][r], l = row_l[buf][r];
            ok = ok && mbar_wait_bounded(&bars.o_full, (uint32_t) (i & 1), status);
            if (!__all_sync(0xffffffffu, ok)) break;
            tc_fence_after();
            const float inv = l > 0.0f ? 1.0f / l : 0.0f;
            uint32_t pk[HEAD_DIM / 2];
            #pragma unroll
            for (int c0v = 0; c0v < HEAD_DIM; c0v += 64) {
                uint32_t v[2][32];
                tmem_ld32(tmem + lane_base + PA_TMEM_O + (uint32_t) c0v, v[0]);
                tmem_ld32(tmem + lane_base + PA_TMEM_O + (uint32_t) (c0v + 32), v[1]);
                tmem_ld_wait();
                #pragma unroll
                for (int k = 0; k < 32; k++)
                    pk[c0v / 2 + k] = pack_f16x2(__uint_as_float(v[k >> 4][2 * (k & 15)]) * inv,
                                                 __uint_as_float(v[k >> 4][2 * (k & 15) + 1]) * inv);
            }
            tc_fence_before();
            mbar_arrive(&bars.o_empty);
            // row (KV head g, entry c, query head h) of the partials; the chunk's rows are contiguous
            const size_t y0 = ((size_t) g * slots + c0) * GQA_TILE;
            if (qi < nq) *reinterpret_cast<float2 *>(part_ml + (y0 + r) * 2) = make_float2(m, l);
            // slice: row x (lane) holds its 4 16-byte pieces at positions k ^ ((x >> 1) & 3)
            const int swz_w = (lane >> 1) & 3;
            #pragma unroll
            for (int p = 0; p < HEAD_DIM / 32; p++) {       // 32 columns (64 bytes) of every row
                #pragma unroll
                for (int k = 0; k < 4; k++)
                    *reinterpret_cast<uint4 *>(wbuf + lane * 64 + ((k ^ swz_w) << 4)) =
                        make_uint4(pk[16 * p + 4 * k], pk[16 * p + 4 * k + 1], pk[16 * p + 4 * k + 2], pk[16 * p + 4 * k + 3]);
                __syncwarp();
                #pragma unroll
                for (int j = 0; j < 4; j++) {                // rows 8j + lane / 4, piece lane % 4
                    const int x = 8 * j + (lane >> 2), k = lane & 3;
                    const int rr = ew * 32 + x;
                    if ((rr >> 3) < nq)
                        __stcs(reinterpret_cast<uint4 *>(part_o + (y0 + rr) * HEAD_DIM + p * 32) + k,
                               *reinterpret_cast<const uint4 *>(wbuf + x * 64 + ((k ^ ((x >> 1) & 3)) << 4)));
                }
                __syncwarp();
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 0) tmem_dealloc_warp(tmem, PA_TMEM_COLS);
}

// ------------------------------------------------------------------ merge per query
// CTA = query t, warp = head h, lane = 8 dimensions: each slot's partial row (through its entry)
// and weight 2^(m_j - M) l_j go to shared memory, then every row's 512 bytes are read once,
// coalesced.
__global__ void prefill_merge_kernel(DevDesc d, int T, int slots, const int * __restrict__ nsel,
        const int * __restrict__ entry_of, const __half * __restrict__ part_o, const float * __restrict__ part_ml,
        OutSpec outs) {
    extern __shared__ float pm_smem[];                       // [n_head][kb] weights, [n_head][kb] rows
    const int t = blockIdx.x, h = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n = max(0, min(nsel[t], d.kb));
    float * w = pm_smem + h * d.kb;
    int * rows = reinterpret_cast<int *>(pm_smem + d.n_head * d.kb) + h * d.kb;
    const int g = h / d.gqa, hh = h % d.gqa;
    float M = -INFINITY;
    for (int j = lane; j < n; j += 32) {
        const int e = entry_of[(size_t) t * d.kb + j];
        const int row = e < 0 ? -1 : (g * slots + e) * d.gqa + hh;
        rows[j] = row;
        if (row >= 0) M = fmaxf(M, part_ml[(size_t) row * 2]);
    }
    M = warp_max(M);
    const float Mu = M == -INFINITY ? 0.0f : M;
    float Wl = 0.0f;
    for (int j = lane; j < n; j += 32) {
        const int row = rows[j];
        float wj = 0.0f;
        if (row >= 0) {
            const float2 ml = *reinterpret_cast<const float2 *>(part_ml + (size_t) row * 2);
            wj = ml.y * exp2f(ml.x - Mu);
        }
        w[j] = wj;
        Wl += wj;
    }
    #pragma unroll
    for (int o = 16; o > 0; o >>= 1) Wl += __shfl_xor_sync(0xffffffffu, Wl, o);
    __syncwarp();
    float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    const uint4 * src = reinterpret_cast<const uint4 *>(part_o) + lane;
    auto load = [&](int j) -> uint4 {
        const int row = rows[j];
        return row >= 0 ? __ldcs(src + (size_t) row * (HEAD_DIM / 8)) : make_uint4(0, 0, 0, 0);
    };
    auto add = [&](const uint4 & x, float wj) {
        const uint32_t xx[4] = {x.x, x.y, x.z, x.w};
        #pragma unroll
        for (int e = 0; e < 4; e++) {
            const float2 f = __half22float2(*reinterpret_cast<const __half2 *>(&xx[e]));
            acc[2 * e] += wj * f.x;
            acc[2 * e + 1] += wj * f.y;
        }
    };
    int j = 0;
    for (; j + 4 <= n; j += 4) {
        uint4 x[4];
        #pragma unroll
        for (int k = 0; k < 4; k++) x[k] = load(j + k);
        #pragma unroll
        for (int k = 0; k < 4; k++) add(x[k], w[j + k]);
    }
    for (; j < n; j++) add(load(j), w[j]);
    const float inv = Wl > 0.0f ? 1.0f / Wl : 0.0f;
    const size_t off = ((size_t) t * d.n_head + h) * HEAD_DIM + lane * 8;
    out_store4(outs, off, make_float4(acc[0] * inv, acc[1] * inv, acc[2] * inv, acc[3] * inv));
    out_store4(outs, off + 4, make_float4(acc[4] * inv, acc[5] * inv, acc[6] * inv, acc[7] * inv));
}

bool prefill_kv_supported(const DevDesc & d, int T) {
    // partial rows are indexed in int32 (TMA coordinates): T * kb * n_head < 2^31
    const bool types = (d.type_k == QSA_TYPE_Q8_0 && d.type_v == QSA_TYPE_Q8_0) ||
                       (d.type_k == QSA_TYPE_F16 && d.type_v == QSA_TYPE_F16);
    return types && d.ratio == PA_CELLS && d.gqa == GQA_TILE &&
           d.head_dim == HEAD_DIM && d.kb <= (1 << PA_SLOT_SHIFT) && d.n_head <= 32 &&
           (int64_t) T * d.kb * d.n_head < ((int64_t) 1 << 31);
}

namespace {
size_t a256(size_t x) { return (x + 255) & ~(size_t) 255; }

struct PrefillKvLayout {
    size_t cnt, cursor, offsets, entries, entry_of, q16, part_o, part_ml, total;
};
PrefillKvLayout prefill_kv_layout(const DevDesc & d, int T, int n_blocks) {
    PrefillKvLayout L;
    const size_t slots = (size_t) T * d.kb;
    L.cnt = 0;
    L.cursor = L.cnt + a256((size_t) n_blocks * 4);
    L.offsets = L.cursor + a256((size_t) n_blocks * 4);
    L.entries = L.offsets + a256((size_t) (n_blocks + 1) * 4);
    L.entry_of = L.entries + a256(slots * 4);
    L.q16 = L.entry_of + a256(slots * 4);
    L.part_o = L.q16 + a256((size_t) T * d.n_head * HEAD_DIM * 2);
    L.part_ml = L.part_o + a256(slots * d.n_head * HEAD_DIM * 2);
    L.total = L.part_ml + a256(slots * d.n_head * 2 * 4);
    return L;
}

// groups x 8 rows x 256 f16 at `ptr` (rows of 512 bytes) seen as [group][atom][row][64 columns]:
// dims {64 columns, 8 rows (512 B apart), 4 atoms (128 B apart), groups (4 KB apart)}; a box of
// box_groups groups lands as [group][atom][8 rows][128 bytes], 128-byte swizzle
bool encode_groups_map(CUtensorMap * map, void * ptr, uint64_t groups, uint32_t box_groups) {
    encode_tiled_fn enc = tensor_map_encoder();
    if (!enc) return false;
    const cuuint64_t dims[4] = {64, 8, 4, (cuuint64_t) groups};
    const cuuint64_t strides[3] = {(cuuint64_t) HEAD_DIM * 2, 128, (cuuint64_t) PA_QROWS};
    const cuuint32_t box[4] = {64, 8, 4, box_groups};
    const cuuint32_t estr[4] = {1, 1, 1, 1};
    return enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4, ptr, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
               CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// an f16 cache (n_ctx rows of row_bytes) as {64 dims, rows, atoms of 64 dims (128 bytes apart)}: a box
// of 64 rows x 4 atoms is one head's [cell][dim] tile in the 128-byte swizzled layout
bool encode_cache_map_f16(CUtensorMap * map, const void * ptr, int64_t row_bytes, int n_ctx, int n_head_kv) {
    encode_tiled_fn enc = tensor_map_encoder();
    if (!enc) return false;
    const cuuint64_t dims[3] = {64, (cuuint64_t) n_ctx, (cuuint64_t) (4 * n_head_kv)};
    const cuuint64_t strides[2] = {(cuuint64_t) row_bytes, 128};
    const cuuint32_t box[3] = {64, (cuuint32_t) PA_CELLS, 4};
    const cuuint32_t estr[3] = {1, 1, 1};
    return enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<void *>(ptr), dims, strides, box, estr,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// the raw bytes of a q8_0 cache (n_ctx rows of row_bytes) as u16 elements; boxes of one head's
// 272 bytes x 64 rows, no swizzle (rows past n_ctx read as zero)
bool encode_cache_map(CUtensorMap * map, const void * ptr, int64_t row_bytes, int n_ctx) {
    encode_tiled_fn enc = tensor_map_encoder();
    if (!enc) return false;
    const cuuint64_t dims[2] = {(cuuint64_t) (row_bytes / 2), (cuuint64_t) n_ctx};
    const cuuint64_t strides[1] = {(cuuint64_t) row_bytes};
    const cuuint32_t box[2] = {(cuuint32_t) (PA_HEAD_Q8 / 2), (cuuint32_t) PA_CELLS};
    const cuuint32_t estr[2] = {1, 1};
    return enc(map, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, const_cast<void *>(ptr), dims, strides, box, estr,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}
}  // namespace

size_t prefill_kv_workspace(const DevDesc & d, int T, int n_blocks) { return prefill_kv_layout(d, T, n_blocks).total; }

cudaError_t launch_prefill_attn_kv(const DevDesc & d, cudaStream_t st, qsa_layer_cache cache, int n_past0, int T,
                                   const void * q, int q_type, const int * sel, const int * nsel, int n_blocks,
                                   unsigned char * ws, OutSpec outs, uint32_t * status) {
    static std::atomic<uint64_t> attr{0};
    cudaError_t e = once_per_device(attr, [] {
        return cudaFuncSetAttribute(prefill_attn_kv_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, PA_SMEM);
    });
    if (e != cudaSuccess) return e;
    const PrefillKvLayout L = prefill_kv_layout(d, T, n_blocks);
    const size_t slots = (size_t) T * d.kb;
    int * cnt = reinterpret_cast<int *>(ws + L.cnt);
    int * cursor = reinterpret_cast<int *>(ws + L.cursor);
    int * offsets = reinterpret_cast<int *>(ws + L.offsets);
    uint32_t * entries = reinterpret_cast<uint32_t *>(ws + L.entries);
    int * entry_of = reinterpret_cast<int *>(ws + L.entry_of);
    __half * q16 = reinterpret_cast<__half *>(ws + L.q16);
    __half * part_o = reinterpret_cast<__half *>(ws + L.part_o);
    float * part_ml = reinterpret_cast<float *>(ws + L.part_ml);
    CUtensorMap q_map, k_map, v_map;
    if (!encode_groups_map(&q_map, q16, (uint64_t) T * d.n_head_kv, 1) ||
        (d.type_k == QSA_TYPE_F16
             ? !encode_cache_map_f16(&k_map, cache.k, d.rb_k, d.n_ctx, d.n_head_kv) ||
               !encode_cache_map_f16(&v_map, cache.v, d.rb_v, d.n_ctx, d.n_head_kv)
             : !encode_cache_map(&k_map, cache.k, d.rb_k, d.n_ctx) || !encode_cache_map(&v_map, cache.v, d.rb_v, d.n_ctx)))
        return cudaErrorNotSupported;
    e = cudaMemsetAsync(cnt, 0, (size_t) n_blocks * 4, st);
    if (e != cudaSuccess) return e;
    const int nthr = 256;
    const unsigned nb_slots = (unsigned) ((slots + nthr - 1) / nthr);
    const int64_t n8 = (int64_t) T * d.n_head * HEAD_DIM / 8;
    prefill_q16_kernel<<<(unsigned) ((n8 + nthr - 1) / nthr), nthr, 0, st>>>(q, q_type, n8, reinterpret_cast<uint4 *>(q16));
    prefill_bucket_count_kernel<<<nb_slots, nthr, 0, st>>>(d, T, sel, nsel, n_blocks, cnt);
    prefill_bucket_scan_kernel<<<1, 1024, 0, st>>>(cnt, n_blocks, offsets, cursor);
    prefill_bucket_fill_kernel<<<nb_slots, nthr, 0, st>>>(d, T, sel, nsel, n_blocks, cursor, entries, entry_of);
    prefill_attn_kv_kernel<<<dim3((unsigned) n_blocks, (unsigned) d.n_head_kv), PA_THREADS, PA_SMEM, st>>>(
        q_map, k_map, v_map, d, n_past0, n_past0 + T, (int) slots, entries, offsets, part_o, part_ml, status);
    const size_t merge_smem = (size_t) d.n_head * d.kb * 8;
    if (merge_smem > 48 * 1024) {
        e = cudaFuncSetAttribute(prefill_merge_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int) merge_smem);
        if (e != cudaSuccess) return e;
    }
    prefill_merge_kernel<<<(unsigned) T, 32 * d.n_head, merge_smem, st>>>(d, T, (int) slots, nsel, entry_of, part_o,
                                                                          part_ml, outs);
    return cudaGetLastError();
}

}  // namespace qsa
