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
//      (counting sort: counts, one scan, a fill); prefill_q16_kernel converts Q to f16 rows;
//   2. prefill_attn_kv_kernel, CTA = (block, KV head): the block's K and V rows of that head are
//      dequantised once into shared memory (f16 of d x q, the rounding of the reference's decode
//      gather); then the CTA walks its queries 16 at a time (16 x 8 query heads = 128 rows) in a
//      warp-specialised pipeline:
//        warp 8      TMA loads of the 16 queries' Q rows (128-byte swizzle) -> sQ
//        warp 9      one thread issues S = Q K^T (16 tcgen05.mma, M=128, N=64 cells, K=16) into one
//                    of two TMEM S buffers, and O = P V (4 tcgen05.mma, M=128, N=256, K=16) into
//                    TMEM; S of chunk i+1 is issued before O of chunk i
//        warps 0-3   thread = row = TMEM lane: S from TMEM, mask of the cells past the query,
//                    P = 2^(s - m) (f16) -> sP, row maximum and sum -> shared memory
//        warps 4-7   thread = row: O from TMEM, O / l (f16) -> swizzled staging in shared memory,
//                    then TMA tensor stores of the rows (query t, slot j, head) to the partials,
//                    and (m, l) of the row
//   3. prefill_merge_kernel: per query, a warp per head merges its slots' partials (log-sum-exp).
// Operands are K-major with the 128-byte swizzle: Q [128 rows][256 dims], K [64 cells][256 dims],
// V^T [256 dims][64 cells], P [128 rows][64 cells]; the O staging has Q's layout.
#include <cuda.h>          // CUtensorMap and its enums; the encoder is reached through the runtime

#include "qsa_kernels.cuh"
#include "qsa_tc.cuh"

namespace qsa {

constexpr int PA_THREADS = 320;                    // warps 0-3 softmax, 4-7 epilogue, 8 loads, 9 MMA
constexpr int PA_QC = 16;                          // queries per chunk
constexpr int PA_ROWS = PA_QC * GQA_TILE;          // 128 MMA rows
constexpr int PA_CELLS = 64;                       // cells of a block (ratio 64)
constexpr int PA_SQ = PA_ROWS * HEAD_DIM * 2;      // 64 KB
constexpr int PA_SK = PA_CELLS * HEAD_DIM * 2;     // 32 KB
constexpr int PA_SV = HEAD_DIM * PA_CELLS * 2;     // 32 KB
constexpr int PA_SP = PA_ROWS * PA_CELLS * 2;      // 16 KB
constexpr int PA_SO = PA_ROWS * HEAD_DIM * 2;      // 64 KB of O staging
constexpr int PA_SMEM = PA_SQ + PA_SK + PA_SV + PA_SP + PA_SO + 1024;
constexpr int PA_ATOM_Q = PA_ROWS * 128;           // bytes of one 64-column atom of sQ / sO
constexpr uint32_t PA_TMEM_COLS = 512;             // S buffers: columns 0..63, 64..127; O: 256..511
constexpr uint32_t PA_TMEM_O = 256;
constexpr uint32_t PA_IDESC_S = umma_idesc_f16(PA_ROWS, PA_CELLS);
constexpr uint32_t PA_IDESC_O = umma_idesc_f16(PA_ROWS, HEAD_DIM);
constexpr int PA_SLOT_SHIFT = 10;                  // entry = query << 10 | slot (slot < MAX_KB)
constexpr int PA_BOX_BYTES = 8 * 128;              // a TMA box: 8 rows x 64 f16

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

__global__ void prefill_bucket_fill_kernel(const DevDesc d, int T, const int * __restrict__ sel,
                                           const int * __restrict__ nsel, int n_blocks, int * __restrict__ cursor,
                                           uint32_t * __restrict__ entries) {
    const int64_t i = (int64_t) blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (int64_t) T * d.kb) return;
    const int t = (int) (i / d.kb), j = (int) (i % d.kb);
    if (j >= nsel[t]) return;
    const int b = sel[i];
    if (b < 0 || b >= n_blocks) return;
    entries[atomicAdd(&cursor[b], 1)] = ((uint32_t) t << PA_SLOT_SHIFT) | (uint32_t) j;
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

// ------------------------------------------------------------------ TMA (tensor maps) and bulk groups
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap * map, int x, int y, uint64_t * bar) {
    asm volatile("cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
                 :: "r"(dst), "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void tma_store_2d(const CUtensorMap * map, int x, int y, uint32_t src) {
    asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.tile.bulk_group [%0, {%1, %2}], [%3];"
                 :: "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(src) : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_read_all() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }
__device__ __forceinline__ void epilogue_sync() { asm volatile("bar.sync 1, 128;" ::: "memory"); }
// barrier of the 128 epilogue threads that also ANDs `ok` over them, so that all leave together
__device__ __forceinline__ bool epilogue_all(bool ok) {
    uint32_t r;
    asm volatile("{\n\t.reg .pred p, q;\n\t"
                 "setp.ne.u32 p, %1, 0;\n\t"
                 "bar.red.and.pred q, 1, 128, p;\n\t"
                 "selp.u32 %0, 1, 0, q;\n\t}"
                 : "=r"(r) : "r"(ok ? 1u : 0u) : "memory");
    return r != 0;
}

// ------------------------------------------------------------------ attention per (block, KV head)
__device__ __forceinline__ uint32_t f16x2_scaled(int8_t a, int8_t b, float d) {
    return pack_f16x2((float) a * d, (float) b * d);        // f16(d x q), exact product rounded once
}

struct PaBarriers {
    uint64_t q_full, q_empty;         // sQ loaded (TMA bytes) / read by the S MMAs (commit)
    uint64_t s_full[2], s_empty[2];   // S buffer written (commit) / read by the 128 softmax threads
    uint64_t p_full, p_empty;         // sP written by the softmax threads / read by the O MMAs (commit)
    uint64_t o_full, o_empty;         // O in TMEM (commit) / read by the 128 epilogue threads
    uint64_t meta_full[2];            // row statistics of a chunk written by the softmax threads
    uint64_t mma_done;                // the MMA thread's last commit before TMEM is released
};

__global__ void __launch_bounds__(PA_THREADS, 1) prefill_attn_kv_kernel(
        const __grid_constant__ CUtensorMap q_map, const __grid_constant__ CUtensorMap o_map, DevDesc d,
        qsa_layer_cache cache, int n_past0, int n_kv, const uint32_t * __restrict__ entries,
        const int * __restrict__ offsets, float * __restrict__ part_ml, uint32_t * __restrict__ status) {
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
    unsigned char * sK = pa_smem_raw + (base - raw) + PA_SQ;
    unsigned char * sV = sK + PA_SK;                        // V^T [256 dims][64 cells]
    unsigned char * sP = sV + PA_SV;
    unsigned char * sO = sP + PA_SP;
    const uint32_t aQ = base, aK = base + PA_SQ, aV = aK + PA_SK, aP = aV + PA_SV, aO = aP + PA_SP;

    if (warp == 0) tmem_alloc_warp(&tmem_slot, PA_TMEM_COLS);
    if (tid == 32) {
        mbar_init(&bars.q_full, 1);
        mbar_init(&bars.q_empty, 1);
        for (int k = 0; k < 2; k++) {
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
    // the loader issues the first chunk's Q rows before the dequantisation below
    auto load_q = [&](int i) {
        const int c0 = e0 + i * PA_QC, nq = min(PA_QC, e1 - c0);
        if (lane == 0) mbar_arrive_expect_tx(&bars.q_full, (uint32_t) (nq * 4 * PA_BOX_BYTES));
        __syncwarp();
        if (lane < nq) {
            const int t = (int) (entries[c0 + lane] >> PA_SLOT_SHIFT);
            const int y = t * d.n_head + g * d.gqa;
            #pragma unroll
            for (int a = 0; a < 4; a++) tma_load_2d(aQ + a * PA_ATOM_Q + lane * PA_BOX_BYTES, &q_map, a * 64, y, &bars.q_full);
        }
    };
    if (warp == 8) load_q(0);

    // ---- K and V of head g of block b -> f16 (d x q), K as [cell][dim], V as [dim][cell]; cells at
    // or past n_kv were never written (their bytes may decode to Inf or NaN, and a masked P of 0
    // times a NaN of V is NaN in the MMA), so they are zero
    const int n_valid = min(PA_CELLS, n_kv - b * PA_CELLS);
    const uint8_t * krow0 = (const uint8_t *) cache.k + (size_t) b * PA_CELLS * d.rb_k + (size_t) g * d.hb_k;
    const uint8_t * vrow0 = (const uint8_t *) cache.v + (size_t) b * PA_CELLS * d.rb_v + (size_t) g * d.hb_v;
    for (int i = tid; i < PA_CELLS * (HEAD_DIM / 8); i += PA_THREADS) {      // (cell, 8-dim group)
        const int cell = i >> 5, d8 = i & 31;
        uint4 w = make_uint4(0, 0, 0, 0);
        if (cell < n_valid) {
            const uint8_t * blk = krow0 + (size_t) cell * d.rb_k + (d8 >> 2) * Q8_0_BYTES;
            const float sc = f16_bits_to_f32(*reinterpret_cast<const uint16_t *>(blk));
            const int8_t * qs = reinterpret_cast<const int8_t *>(blk + 2) + (d8 & 3) * 8;
            w.x = f16x2_scaled(qs[0], qs[1], sc); w.y = f16x2_scaled(qs[2], qs[3], sc);
            w.z = f16x2_scaled(qs[4], qs[5], sc); w.w = f16x2_scaled(qs[6], qs[7], sc);
        }
        *reinterpret_cast<uint4 *>(sK + sw128_off(PA_CELLS, cell, d8 * 8)) = w;
    }
    for (int i = tid; i < (HEAD_DIM / 8) * (PA_CELLS / 8); i += PA_THREADS) {   // (8-dim group, 8-cell group)
        const int d8 = i >> 3, c8 = i & 7;
        uint16_t val[8][8];                                   // [dim][cell]
        #pragma unroll
        for (int c = 0; c < 8; c++) {
            if (c8 * 8 + c < n_valid) {
                const uint8_t * blk = vrow0 + (size_t) (c8 * 8 + c) * d.rb_v + (d8 >> 2) * Q8_0_BYTES;
                const float sc = f16_bits_to_f32(*reinterpret_cast<const uint16_t *>(blk));
                const int8_t * qs = reinterpret_cast<const int8_t *>(blk + 2) + (d8 & 3) * 8;
                #pragma unroll
                for (int k = 0; k < 8; k++) val[k][c] = f32_to_f16_bits((float) qs[k] * sc);
            } else {
                #pragma unroll
                for (int k = 0; k < 8; k++) val[k][c] = 0;
            }
        }
        #pragma unroll
        for (int k = 0; k < 8; k++) {
            uint4 w;
            w.x = val[k][0] | ((uint32_t) val[k][1] << 16); w.y = val[k][2] | ((uint32_t) val[k][3] << 16);
            w.z = val[k][4] | ((uint32_t) val[k][5] << 16); w.w = val[k][6] | ((uint32_t) val[k][7] << 16);
            *reinterpret_cast<uint4 *>(sV + sw128_off(HEAD_DIM, d8 * 8 + k, c8 * 8)) = w;
        }
    }
    fence_async_smem();                                     // K and V tiles visible to the tensor core
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tmem_slot;

    if (warp == 8) {
        // ---------------------------------------------------------------- Q loads
        int i = 1;
        for (; i < n_chunks; i++) {
            if (!mbar_wait_bounded(&bars.q_empty, (uint32_t) ((i - 1) & 1), status)) break;   // S MMAs of i-1 done
            load_q(i);
        }
        // every issued load has landed before the CTA can leave
        mbar_wait_bounded(&bars.q_full, (uint32_t) ((i - 1) & 1), status);
    } else if (warp == 9) {
        // ---------------------------------------------------------------- MMA issue (one thread)
        if (lane == 0) {
            bool ok = true;
            auto issue_s = [&](int i) {
                const int buf = i & 1;
                ok = ok && mbar_wait_bounded(&bars.q_full, (uint32_t) (i & 1), status);
                if (i >= 2) ok = ok && mbar_wait_bounded(&bars.s_empty[buf], (uint32_t) (((i - 2) >> 1) & 1), status);
                if (!ok) return;
                tc_fence_after();
                #pragma unroll
                for (int kk = 0; kk < HEAD_DIM / 16; kk++)
                    umma_f16(tmem + (uint32_t) (buf * PA_CELLS),
                             umma_desc_sw128(aQ + (kk >> 2) * PA_ATOM_Q + (kk & 3) * 32),
                             umma_desc_sw128(aK + (kk >> 2) * (PA_CELLS * 128) + (kk & 3) * 32), PA_IDESC_S, kk > 0);
                umma_commit(&bars.s_full[buf]);
                umma_commit(&bars.q_empty);
            };
            issue_s(0);
            for (int i = 0; i < n_chunks && ok; i++) {
                if (i + 1 < n_chunks) issue_s(i + 1);
                ok = ok && mbar_wait_bounded(&bars.p_full, (uint32_t) (i & 1), status);
                if (i >= 1) ok = ok && mbar_wait_bounded(&bars.o_empty, (uint32_t) ((i - 1) & 1), status);
                if (!ok) break;
                tc_fence_after();
                #pragma unroll
                for (int kk = 0; kk < PA_CELLS / 16; kk++)
                    umma_f16(tmem + PA_TMEM_O, umma_desc_sw128(aP + kk * 32), umma_desc_sw128(aV + kk * 32), PA_IDESC_O, kk > 0);
                umma_commit(&bars.o_full);
                umma_commit(&bars.p_empty);
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
            const int buf = i & 1, c0 = e0 + i * PA_QC, nq = min(PA_QC, e1 - c0);
            if (!mbar_wait_bounded(&bars.s_full[buf], (uint32_t) ((i >> 1) & 1), status)) break;
            tc_fence_after();
            uint32_t v[32], u[32];
            tmem_ld32(tmem + lane_base + (uint32_t) (buf * PA_CELLS), v);
            tmem_ld32(tmem + lane_base + (uint32_t) (buf * PA_CELLS + 32), u);
            tmem_ld_wait();
            tc_fence_before();
            mbar_arrive(&bars.s_empty[buf]);
            int lim = -1;                                     // cells 0..lim of the block are visible
            if (qi < nq) lim = n_past0 + (int) (entries[c0 + qi] >> PA_SLOT_SHIFT) - b * PA_CELLS;
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
        const int r = tid - 128, qi = r >> 3, h = r & 7;
        const uint32_t lane_base = (uint32_t) ((warp - 4) * 32) << 16;
        for (int i = 0; i < n_chunks; i++) {
            const int buf = i & 1, c0 = e0 + i * PA_QC, nq = min(PA_QC, e1 - c0);
            bool ok = mbar_wait_bounded(&bars.meta_full[buf], (uint32_t) ((i >> 1) & 1), status);
            const float m = row_m[buf][r], l = row_l[buf][r];
            ok = ok && mbar_wait_bounded(&bars.o_full, (uint32_t) (i & 1), status);
            if (r < PA_QC) bulk_wait_read_all();              // this thread's stores of chunk i-1 have read sO
            if (!epilogue_all(ok)) break;
            tc_fence_after();
            const float inv = l > 0.0f ? 1.0f / l : 0.0f;
            #pragma unroll 1
            for (int c0v = 0; c0v < HEAD_DIM; c0v += 32) {
                uint32_t v[32];
                tmem_ld32(tmem + lane_base + PA_TMEM_O + (uint32_t) c0v, v);
                tmem_ld_wait();
                #pragma unroll
                for (int k = 0; k < 4; k++)
                    *reinterpret_cast<uint4 *>(sO + sw128_off(PA_ROWS, r, c0v + 8 * k)) =
                        make_uint4(pack_f16x2(__uint_as_float(v[8 * k]) * inv, __uint_as_float(v[8 * k + 1]) * inv),
                                   pack_f16x2(__uint_as_float(v[8 * k + 2]) * inv, __uint_as_float(v[8 * k + 3]) * inv),
                                   pack_f16x2(__uint_as_float(v[8 * k + 4]) * inv, __uint_as_float(v[8 * k + 5]) * inv),
                                   pack_f16x2(__uint_as_float(v[8 * k + 6]) * inv, __uint_as_float(v[8 * k + 7]) * inv));
            }
            tc_fence_before();
            mbar_arrive(&bars.o_empty);
            if (qi < nq) {
                const uint32_t e = entries[c0 + qi];
                const size_t slot = ((size_t) (e >> PA_SLOT_SHIFT) * d.kb + (e & ((1u << PA_SLOT_SHIFT) - 1))) * d.n_head +
                                    g * d.gqa + h;
                *reinterpret_cast<float2 *>(part_ml + slot * 2) = make_float2(m, l);
            }
            fence_async_smem();                               // staging visible to the TMA unit
            epilogue_sync();
            if (r < nq) {                                     // thread q stores query q's 8 rows
                const uint32_t e = entries[c0 + r];
                const int y = (int) (((e >> PA_SLOT_SHIFT) * (uint32_t) d.kb + (e & ((1u << PA_SLOT_SHIFT) - 1))) *
                                     (uint32_t) d.n_head) + g * d.gqa;
                #pragma unroll
                for (int a = 0; a < 4; a++) tma_store_2d(&o_map, a * 64, y, aO + a * PA_ATOM_Q + r * PA_BOX_BYTES);
                bulk_commit();
            }
        }
        if (r < PA_QC) bulk_wait_all();                       // the partials are written before the CTA ends
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (warp == 0) tmem_dealloc_warp(tmem, PA_TMEM_COLS);
}

// ------------------------------------------------------------------ merge per query
// CTA = query t, warp = head h, lane = 8 dimensions: the weights 2^(m_j - M) l_j of the slots go
// to shared memory, then every slot's 512-byte partial row is read once, coalesced.
__global__ void prefill_merge_kernel(DevDesc d, int T, const int * __restrict__ nsel,
        const __half * __restrict__ part_o, const float * __restrict__ part_ml, float * __restrict__ out) {
    extern __shared__ float pm_w[];                          // [n_head][kb]
    const int t = blockIdx.x, h = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n = max(0, min(nsel[t], d.kb));
    float * w = pm_w + h * d.kb;
    float M = -INFINITY;
    for (int j = lane; j < n; j += 32) M = fmaxf(M, part_ml[(((size_t) t * d.kb + j) * d.n_head + h) * 2]);
    M = warp_max(M);
    const float Mu = M == -INFINITY ? 0.0f : M;
    float Wl = 0.0f;
    for (int j = lane; j < n; j += 32) {
        const float2 ml = *reinterpret_cast<const float2 *>(part_ml + (((size_t) t * d.kb + j) * d.n_head + h) * 2);
        const float wj = ml.y * exp2f(ml.x - Mu);
        w[j] = wj;
        Wl += wj;
    }
    #pragma unroll
    for (int o = 16; o > 0; o >>= 1) Wl += __shfl_xor_sync(0xffffffffu, Wl, o);
    __syncwarp();
    float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    const uint4 * src = reinterpret_cast<const uint4 *>(part_o + ((size_t) t * d.kb * d.n_head + h) * HEAD_DIM) + lane;
    const size_t jstride = (size_t) d.n_head * HEAD_DIM / 8;   // uint4 per slot
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
        for (int k = 0; k < 4; k++) x[k] = __ldcs(src + (size_t) (j + k) * jstride);
        #pragma unroll
        for (int k = 0; k < 4; k++) add(x[k], w[j + k]);
    }
    for (; j < n; j++) add(__ldcs(src + (size_t) j * jstride), w[j]);
    const float inv = Wl > 0.0f ? 1.0f / Wl : 0.0f;
    float4 * dst = reinterpret_cast<float4 *>(out + ((size_t) t * d.n_head + h) * HEAD_DIM) + lane * 2;
    dst[0] = make_float4(acc[0] * inv, acc[1] * inv, acc[2] * inv, acc[3] * inv);
    dst[1] = make_float4(acc[4] * inv, acc[5] * inv, acc[6] * inv, acc[7] * inv);
}

bool prefill_kv_supported(const DevDesc & d) {
    return d.type_k == QSA_TYPE_Q8_0 && d.type_v == QSA_TYPE_Q8_0 && d.ratio == PA_CELLS && d.gqa == GQA_TILE &&
           d.kb <= (1 << PA_SLOT_SHIFT) && d.n_head <= 32;
}

namespace {
size_t a256(size_t x) { return (x + 255) & ~(size_t) 255; }

struct PrefillKvLayout {
    size_t cnt, cursor, offsets, entries, q16, part_o, part_ml, total;
};
PrefillKvLayout prefill_kv_layout(const DevDesc & d, int T, int n_blocks) {
    PrefillKvLayout L;
    const size_t slots = (size_t) T * d.kb;
    L.cnt = 0;
    L.cursor = L.cnt + a256((size_t) n_blocks * 4);
    L.offsets = L.cursor + a256((size_t) n_blocks * 4);
    L.entries = L.offsets + a256((size_t) (n_blocks + 1) * 4);
    L.q16 = L.entries + a256(slots * 4);
    L.part_o = L.q16 + a256((size_t) T * d.n_head * HEAD_DIM * 2);
    L.part_ml = L.part_o + a256(slots * d.n_head * HEAD_DIM * 2);
    L.total = L.part_ml + a256(slots * d.n_head * 2 * 4);
    return L;
}

// cuTensorMapEncodeTiled, reached through the runtime's driver entry-point query
typedef CUresult (*encode_tiled_fn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                    const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                    CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
encode_tiled_fn tensor_map_encoder() {
    static encode_tiled_fn fn = nullptr;
    if (!fn) {
        void * f = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<encode_tiled_fn>(f);
    }
    return fn;
}

// rows x 256 f16 at `ptr` (rows of 512 bytes), boxes of 8 rows x 64 columns, 128-byte swizzle
bool encode_rows_map(CUtensorMap * map, void * ptr, uint64_t rows) {
    encode_tiled_fn enc = tensor_map_encoder();
    if (!enc) return false;
    const cuuint64_t dims[2] = {(cuuint64_t) HEAD_DIM, (cuuint64_t) rows};
    const cuuint64_t strides[1] = {(cuuint64_t) HEAD_DIM * 2};
    const cuuint32_t box[2] = {64, 8};
    const cuuint32_t estr[2] = {1, 1};
    return enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, ptr, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
               CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}
}  // namespace

size_t prefill_kv_workspace(const DevDesc & d, int T, int n_blocks) { return prefill_kv_layout(d, T, n_blocks).total; }

cudaError_t launch_prefill_attn_kv(const DevDesc & d, cudaStream_t st, qsa_layer_cache cache, int n_past0, int T,
                                   const void * q, int q_type, const int * sel, const int * nsel, int n_blocks,
                                   unsigned char * ws, float * out, uint32_t * status) {
    static bool attr = false;
    if (!attr) {
        cudaError_t e = cudaFuncSetAttribute(prefill_attn_kv_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, PA_SMEM);
        if (e != cudaSuccess) return e;
        attr = true;
    }
    const PrefillKvLayout L = prefill_kv_layout(d, T, n_blocks);
    const size_t slots = (size_t) T * d.kb;
    int * cnt = reinterpret_cast<int *>(ws + L.cnt);
    int * cursor = reinterpret_cast<int *>(ws + L.cursor);
    int * offsets = reinterpret_cast<int *>(ws + L.offsets);
    uint32_t * entries = reinterpret_cast<uint32_t *>(ws + L.entries);
    __half * q16 = reinterpret_cast<__half *>(ws + L.q16);
    __half * part_o = reinterpret_cast<__half *>(ws + L.part_o);
    float * part_ml = reinterpret_cast<float *>(ws + L.part_ml);
    CUtensorMap q_map, o_map;
    if (!encode_rows_map(&q_map, q16, (uint64_t) T * d.n_head) || !encode_rows_map(&o_map, part_o, (uint64_t) slots * d.n_head))
        return cudaErrorNotSupported;
    cudaError_t e = cudaMemsetAsync(cnt, 0, (size_t) n_blocks * 4, st);
    if (e != cudaSuccess) return e;
    const int nthr = 256;
    const unsigned nb_slots = (unsigned) ((slots + nthr - 1) / nthr);
    const int64_t n8 = (int64_t) T * d.n_head * HEAD_DIM / 8;
    prefill_q16_kernel<<<(unsigned) ((n8 + nthr - 1) / nthr), nthr, 0, st>>>(q, q_type, n8, reinterpret_cast<uint4 *>(q16));
    prefill_bucket_count_kernel<<<nb_slots, nthr, 0, st>>>(d, T, sel, nsel, n_blocks, cnt);
    prefill_bucket_scan_kernel<<<1, 1024, 0, st>>>(cnt, n_blocks, offsets, cursor);
    prefill_bucket_fill_kernel<<<nb_slots, nthr, 0, st>>>(d, T, sel, nsel, n_blocks, cursor, entries);
    prefill_attn_kv_kernel<<<dim3((unsigned) n_blocks, (unsigned) d.n_head_kv), PA_THREADS, PA_SMEM, st>>>(
        q_map, o_map, d, cache, n_past0, n_past0 + T, entries, offsets, part_ml, status);
    const size_t merge_smem = (size_t) d.n_head * d.kb * 4;
    if (merge_smem > 48 * 1024) {
        e = cudaFuncSetAttribute(prefill_merge_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int) merge_smem);
        if (e != cudaSuccess) return e;
    }
    prefill_merge_kernel<<<(unsigned) T, 32 * d.n_head, merge_smem, st>>>(d, T, nsel, part_o, part_ml, out);
    return cudaGetLastError();
}

}  // namespace qsa
