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
//      (counting sort: counts, one scan, a fill);
//   2. prefill_attn_kv_kernel, CTA = (block, KV head): the block's K and V rows of that head are
//      dequantised once into shared memory (f16 of d x q, the rounding of the reference's decode
//      gather), then, 16 queries at a time (16 x 8 query heads = 128 rows), S = Q K^T runs as 16
//      tcgen05.mma (M=128, N=64 cells, K=16) into TMEM; one thread per row takes S from TMEM,
//      masks the cells past its query, and writes P = 2^(s - m) (f16) to shared memory;
//      O = P V runs as 4 tcgen05.mma (M=128, N=256 dims, K=16 cells) into TMEM; each row thread
//      stores O / l (f16) with (m, l) as the partial state of (query, slot, head);
//   3. prefill_merge_kernel: per (query, head), the log-sum-exp merge of its slots' partials.
// Operands are K-major with the 128-byte swizzle: Q [128 rows][256 dims], K [64 cells][256 dims],
// V^T [256 dims][64 cells], P [128 rows][64 cells].
#include "qsa_kernels.cuh"
#include "qsa_tc.cuh"

namespace qsa {

constexpr int PA_THREADS = 256;
constexpr int PA_QC = 16;                          // queries per chunk
constexpr int PA_ROWS = PA_QC * GQA_TILE;          // 128 MMA rows
constexpr int PA_CELLS = 64;                       // cells of a block (ratio 64)
constexpr int PA_SQ = PA_ROWS * HEAD_DIM * 2;      // 64 KB
constexpr int PA_SK = PA_CELLS * HEAD_DIM * 2;     // 32 KB
constexpr int PA_SV = HEAD_DIM * PA_CELLS * 2;     // 32 KB
constexpr int PA_SP = PA_ROWS * PA_CELLS * 2;      // 16 KB
constexpr int PA_SMEM = PA_SQ + PA_SK + PA_SV + PA_SP + 1024;
constexpr uint32_t PA_TMEM_COLS = 512;             // S: columns 0..63, O: columns 256..511
constexpr uint32_t PA_IDESC_S = umma_idesc_f16(PA_ROWS, PA_CELLS);
constexpr uint32_t PA_IDESC_O = umma_idesc_f16(PA_ROWS, HEAD_DIM);
constexpr int PA_SLOT_SHIFT = 10;                  // entry = query << 10 | slot (slot < MAX_KB)

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

// ------------------------------------------------------------------ attention per (block, KV head)
__device__ __forceinline__ uint32_t f16x2_scaled(int8_t a, int8_t b, float d) {
    return pack_f16x2((float) a * d, (float) b * d);        // f16(d x q), exact product rounded once
}

__global__ void __launch_bounds__(PA_THREADS, 1) prefill_attn_kv_kernel(DevDesc d, qsa_layer_cache cache, int n_past0, int n_kv,
        const void * __restrict__ q, int q_type, const uint32_t * __restrict__ entries, const int * __restrict__ offsets,
        __half * __restrict__ part_o, float * __restrict__ part_ml, uint32_t * __restrict__ status) {
    extern __shared__ __align__(1024) unsigned char pa_smem_raw[];
    __shared__ uint64_t mma_bar;
    __shared__ uint32_t tmem_slot;
    const int b = blockIdx.x, g = blockIdx.y;
    const int e0 = offsets[b], e1 = offsets[b + 1];
    if (e0 >= e1) return;                                   // no query selected this block
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const uint32_t raw = smem_u32(pa_smem_raw);
    const uint32_t base = (raw + 1023u) & ~1023u;
    unsigned char * sQ = pa_smem_raw + (base - raw);
    unsigned char * sK = sQ + PA_SQ;
    unsigned char * sV = sK + PA_SK;                        // V^T [256 dims][64 cells]
    unsigned char * sP = sV + PA_SV;
    const uint32_t aQ = base, aK = base + PA_SQ, aV = aK + PA_SK, aP = aV + PA_SV;

    if (warp == 0) tmem_alloc_warp(&tmem_slot, PA_TMEM_COLS);
    if (tid == 0) {
        mbar_init(&mma_bar, 1);
        fence_mbar_init();
    }
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
    uint32_t phase = 0;
    bool ok = true;
    for (int c0 = e0; c0 < e1; c0 += PA_QC) {
        const int nq = min(PA_QC, e1 - c0);
        // ---- Q rows (query qi, head h of group g) -> f16
        for (int i = tid; i < PA_ROWS * (HEAD_DIM / 8); i += PA_THREADS) {
            const int r = i >> 5, d8 = i & 31, qi = r >> 3, h = r & 7;
            uint4 w = make_uint4(0, 0, 0, 0);
            if (qi < nq && h < d.gqa) {
                const int t = (int) (entries[c0 + qi] >> PA_SLOT_SHIFT);
                const size_t o = ((size_t) t * d.n_head + g * d.gqa + h) * HEAD_DIM + d8 * 8;
                float f[8];
                if (q_type == QSA_TYPE_BF16) {
                    const uint4 x = *reinterpret_cast<const uint4 *>(reinterpret_cast<const __nv_bfloat16 *>(q) + o);
                    const uint32_t xx[4] = {x.x, x.y, x.z, x.w};
                    #pragma unroll
                    for (int k = 0; k < 4; k++) { f[2 * k] = __uint_as_float(xx[k] << 16); f[2 * k + 1] = __uint_as_float(xx[k] & 0xffff0000u); }
                } else {
                    const float4 x0 = *reinterpret_cast<const float4 *>(reinterpret_cast<const float *>(q) + o);
                    const float4 x1 = *reinterpret_cast<const float4 *>(reinterpret_cast<const float *>(q) + o + 4);
                    f[0] = x0.x; f[1] = x0.y; f[2] = x0.z; f[3] = x0.w; f[4] = x1.x; f[5] = x1.y; f[6] = x1.z; f[7] = x1.w;
                }
                w.x = pack_f16x2(f[0], f[1]); w.y = pack_f16x2(f[2], f[3]);
                w.z = pack_f16x2(f[4], f[5]); w.w = pack_f16x2(f[6], f[7]);
            }
            *reinterpret_cast<uint4 *>(sQ + sw128_off(PA_ROWS, r, d8 * 8)) = w;
        }
        fence_async_smem();
        tc_fence_before();
        __syncthreads();
        tc_fence_after();
        if (tid == 0) {                                       // S = Q K^T: 16 k-steps of 16 dims
            #pragma unroll
            for (int kk = 0; kk < HEAD_DIM / 16; kk++)
                umma_f16(tmem, umma_desc_sw128(aQ + (kk >> 2) * (PA_ROWS * 128) + (kk & 3) * 32),
                         umma_desc_sw128(aK + (kk >> 2) * (PA_CELLS * 128) + (kk & 3) * 32), PA_IDESC_S, kk > 0);
            umma_commit(&mma_bar);
        }
        ok = mbar_wait_bounded(&mma_bar, phase, status) && ok;
        phase ^= 1u;
        tc_fence_after();
        // ---- softmax of each row over the block's cells (thread = row = TMEM lane)
        float row_m = 0.0f, row_l = 0.0f;
        int row_t = -1, row_j = 0;
        if (warp < 4) {
            const int r = warp * 32 + lane, qi = r >> 3, h = r & 7;
            uint32_t v[32], u[32];
            tmem_ld32(tmem + ((uint32_t) (warp * 32) << 16) + 0u, v);
            tmem_ld32(tmem + ((uint32_t) (warp * 32) << 16) + 32u, u);
            tmem_ld_wait();
            int qpos = -1;
            if (qi < nq && h < d.gqa) {
                const uint32_t e = entries[c0 + qi];
                row_t = (int) (e >> PA_SLOT_SHIFT);
                row_j = (int) (e & ((1u << PA_SLOT_SHIFT) - 1));
                qpos = n_past0 + row_t;
            }
            const int lim = qpos - b * PA_CELLS;              // cells 0..lim are visible
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
            #pragma unroll
            for (int c8 = 0; c8 < 8; c8++)
                *reinterpret_cast<uint4 *>(sP + sw128_off(PA_ROWS, r, c8 * 8)) =
                    make_uint4(pk[4 * c8], pk[4 * c8 + 1], pk[4 * c8 + 2], pk[4 * c8 + 3]);
            row_m = m;
            row_l = l;
        }
        fence_async_smem();
        tc_fence_before();
        __syncthreads();
        tc_fence_after();
        if (tid == 0) {                                       // O = P V: 4 k-steps of 16 cells
            #pragma unroll
            for (int kk = 0; kk < PA_CELLS / 16; kk++)
                umma_f16(tmem + 256u, umma_desc_sw128(aP + kk * 32), umma_desc_sw128(aV + kk * 32), PA_IDESC_O, kk > 0);
            umma_commit(&mma_bar);
        }
        ok = mbar_wait_bounded(&mma_bar, phase, status) && ok;
        phase ^= 1u;
        tc_fence_after();
        if (warp < 4) {
            const int r = warp * 32 + lane, h = r & 7;
            const float inv = row_l > 0.0f ? 1.0f / row_l : 0.0f;
            const bool store = ok && row_t >= 0;
            const size_t slot = ((size_t) row_t * d.kb + row_j) * d.n_head + g * d.gqa + h;
            #pragma unroll 1
            for (int c0v = 0; c0v < HEAD_DIM; c0v += 32) {
                uint32_t v[32];
                tmem_ld32(tmem + ((uint32_t) (warp * 32) << 16) + 256u + (uint32_t) c0v, v);
                tmem_ld_wait();
                if (store) {
                    uint4 * dst = reinterpret_cast<uint4 *>(part_o + slot * HEAD_DIM + c0v);
                    #pragma unroll
                    for (int k = 0; k < 4; k++)
                        dst[k] = make_uint4(pack_f16x2(__uint_as_float(v[8 * k]) * inv, __uint_as_float(v[8 * k + 1]) * inv),
                                            pack_f16x2(__uint_as_float(v[8 * k + 2]) * inv, __uint_as_float(v[8 * k + 3]) * inv),
                                            pack_f16x2(__uint_as_float(v[8 * k + 4]) * inv, __uint_as_float(v[8 * k + 5]) * inv),
                                            pack_f16x2(__uint_as_float(v[8 * k + 6]) * inv, __uint_as_float(v[8 * k + 7]) * inv));
                }
            }
            if (store) *reinterpret_cast<float2 *>(part_ml + slot * 2) = make_float2(row_m, row_l);
        }
        tc_fence_before();
        __syncthreads();                                      // sQ, sP and TMEM are free for the next chunk
        tc_fence_after();
    }
    if (warp == 0) tmem_dealloc_warp(tmem, PA_TMEM_COLS);
}

// ------------------------------------------------------------------ merge per (query, head)
__global__ void __launch_bounds__(HEAD_DIM) prefill_merge_kernel(DevDesc d, int T, const int * __restrict__ nsel,
        const __half * __restrict__ part_o, const float * __restrict__ part_ml, float * __restrict__ out) {
    const int t = blockIdx.x, h = blockIdx.y, dim = threadIdx.x;
    const int n = max(0, min(nsel[t], d.kb));
    float M = -INFINITY;
    for (int j = 0; j < n; j++) M = fmaxf(M, part_ml[(((size_t) t * d.kb + j) * d.n_head + h) * 2]);
    const float Mu = M == -INFINITY ? 0.0f : M;
    float W = 0.0f, acc = 0.0f;
    for (int j = 0; j < n; j++) {
        const size_t slot = ((size_t) t * d.kb + j) * d.n_head + h;
        const float2 ml = *reinterpret_cast<const float2 *>(part_ml + slot * 2);
        const float w = ml.y * exp2f(ml.x - Mu);
        W += w;
        acc += w * __half2float(part_o[slot * HEAD_DIM + dim]);
    }
    out[((size_t) t * d.n_head + h) * HEAD_DIM + dim] = W > 0.0f ? acc / W : 0.0f;
}

bool prefill_kv_supported(const DevDesc & d) {
    return d.type_k == QSA_TYPE_Q8_0 && d.type_v == QSA_TYPE_Q8_0 && d.ratio == PA_CELLS && d.gqa == GQA_TILE &&
           d.kb <= (1 << PA_SLOT_SHIFT);
}

size_t prefill_kv_workspace(const DevDesc & d, int T, int n_blocks) {
    auto a256 = [](size_t x) { return (x + 255) & ~(size_t) 255; };
    const size_t slots = (size_t) T * d.kb;
    return a256((size_t) n_blocks * 4) * 2 + a256((size_t) (n_blocks + 1) * 4) + a256(slots * 4) +
           a256(slots * d.n_head * HEAD_DIM * 2) + a256(slots * d.n_head * 2 * 4);
}

cudaError_t launch_prefill_attn_kv(const DevDesc & d, cudaStream_t st, qsa_layer_cache cache, int n_past0, int T,
                                   const void * q, int q_type, const int * sel, const int * nsel, int n_blocks,
                                   unsigned char * ws, float * out, uint32_t * status) {
    static bool attr = false;
    if (!attr) {
        cudaError_t e = cudaFuncSetAttribute(prefill_attn_kv_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, PA_SMEM);
        if (e != cudaSuccess) return e;
        attr = true;
    }
    auto a256 = [](size_t x) { return (x + 255) & ~(size_t) 255; };
    const size_t slots = (size_t) T * d.kb;
    int * cnt = reinterpret_cast<int *>(ws);
    int * cursor = reinterpret_cast<int *>(ws + a256((size_t) n_blocks * 4));
    int * offsets = reinterpret_cast<int *>(ws + 2 * a256((size_t) n_blocks * 4));
    uint32_t * entries = reinterpret_cast<uint32_t *>(ws + 2 * a256((size_t) n_blocks * 4) + a256((size_t) (n_blocks + 1) * 4));
    __half * part_o = reinterpret_cast<__half *>(reinterpret_cast<unsigned char *>(entries) + a256(slots * 4));
    float * part_ml = reinterpret_cast<float *>(reinterpret_cast<unsigned char *>(part_o) + a256(slots * d.n_head * HEAD_DIM * 2));
    cudaError_t e = cudaMemsetAsync(cnt, 0, (size_t) n_blocks * 4, st);
    if (e != cudaSuccess) return e;
    const int nthr = 256;
    const unsigned nb_slots = (unsigned) ((slots + nthr - 1) / nthr);
    prefill_bucket_count_kernel<<<nb_slots, nthr, 0, st>>>(d, T, sel, nsel, n_blocks, cnt);
    prefill_bucket_scan_kernel<<<1, 1024, 0, st>>>(cnt, n_blocks, offsets, cursor);
    prefill_bucket_fill_kernel<<<nb_slots, nthr, 0, st>>>(d, T, sel, nsel, n_blocks, cursor, entries);
    prefill_attn_kv_kernel<<<dim3((unsigned) n_blocks, (unsigned) d.n_head_kv), PA_THREADS, PA_SMEM, st>>>(
        d, cache, n_past0, n_past0 + T, q, q_type, entries, offsets, part_o, part_ml, status);
    prefill_merge_kernel<<<dim3((unsigned) T, (unsigned) d.n_head), HEAD_DIM, 0, st>>>(d, T, nsel, part_o, part_ml, out);
    return cudaGetLastError();
}

}  // namespace qsa
