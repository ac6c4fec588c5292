// qsa_append.cu -- KV append (q8_0/f16 quantisation), raw indexer-key append, pooled-key update.
//
// Reference: the cache writes of graph_builder::sparse_attn_decode (ggml_set_rows,
// src/qwfn_graph.cpp:466-469, 504-528) and sparse_attn/qsa_top_k (ggml_cpy, :249-254, :349-360);
// the pooled key of a block, qsa_pool_blocks (src/qwfn_graph.cpp:412-429), decode use (:470-476),
// post-prefill rebuild qsa_pool_rebuild (:431-448) driven from src/qwfn_engine.cpp:761-798.
#include "qsa_kernels.cuh"

namespace qsa {

// ---------------------------------------------------------------------------------------------
// One q8_0 block (32 values) per warp, lane = element (q8_0_quant_lane).
__device__ __forceinline__ void quantize_q8_0_warp(const float * __restrict__ x, uint8_t * __restrict__ dst, int lane) {
    uint16_t dbits;
    dst[2 + lane] = (uint8_t) q8_0_quant_lane(x[lane], dbits);
    if (lane == 0) *reinterpret_cast<uint16_t *>(dst) = dbits;   // q8_0 blocks are 2-byte aligned
}

// Write one token row of K (or V) with a whole CTA: kv_dim/32 q8_0 blocks, one per warp in turn.
__device__ __forceinline__ void write_kv_row(const DevDesc & d, int type, const float * __restrict__ x,
                                             uint8_t * __restrict__ row, int kv_dim) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    if (type == QSA_TYPE_Q8_0) {
        for (int b = warp; b < kv_dim / QK8_0; b += nw)
            quantize_q8_0_warp(x + b * QK8_0, row + (size_t) b * Q8_0_BYTES, lane);
    } else {
        uint16_t * h = reinterpret_cast<uint16_t *>(row);
        for (int i = threadIdx.x; i < kv_dim; i += blockDim.x) h[i] = f32_to_f16_bits(x[i]);
    }
}

// ---------------------------------------------------------------------------------------------
// Pooled key of block b by one warp; lane owns dims 4*lane .. 4*lane+3 (idx_dim == 128).
// Arithmetic as the oracle restates qsa_pool_blocks: sequential f32 sum of the r member rows,
// times the f32 1/r; sum of squares of f32 products in double, mean rounded to f32,
// scale = 1/sqrtf(mean + eps) (IEEE), times k_norm_w; IMRoPE at position b*r with the angle of
// pair i obtained by i successive f32 multiplies by theta_scale (ggml's cache recurrence), cos and
// sin of that f32 angle (evaluated in double and rounded), NEOX pairs (i, i + rope_dim/2).
// `rows` points at the block's first raw-key row (global memory, or a shared-memory copy).
__device__ void pool_block_warp(const DevDesc & d, const uint16_t * __restrict__ rows, int64_t b,
                                uint16_t * __restrict__ pool_row, float * __restrict__ out_f32) {
    const int lane = threadIdx.x & 31;
    const int r = d.ratio;
    float x[4] = {0.f, 0.f, 0.f, 0.f};
    const uint16_t * base = rows + 4 * lane;
    // rows are fetched 8 at a time (independent loads in flight), then added strictly in order
    for (int i0 = 0; i0 < r; i0 += 8) {
        uint2 w[8];
        #pragma unroll
        for (int k = 0; k < 8; k++)
            w[k] = i0 + k < r ? *reinterpret_cast<const uint2 *>(base + (size_t) (i0 + k) * MAX_IDX_DIM) : make_uint2(0, 0);
        #pragma unroll
        for (int k = 0; k < 8; k++) {
            if (i0 + k >= r) break;
            const float v0 = f16_bits_to_f32((uint16_t) (w[k].x & 0xffff)), v1 = f16_bits_to_f32((uint16_t) (w[k].x >> 16));
            const float v2 = f16_bits_to_f32((uint16_t) (w[k].y & 0xffff)), v3 = f16_bits_to_f32((uint16_t) (w[k].y >> 16));
            if (i0 + k == 0) { x[0] = v0; x[1] = v1; x[2] = v2; x[3] = v3; }
            else { x[0] = __fadd_rn(x[0], v0); x[1] = __fadd_rn(x[1], v1); x[2] = __fadd_rn(x[2], v2); x[3] = __fadd_rn(x[3], v3); }
        }
    }
    double ss = 0.0;
    #pragma unroll
    for (int e = 0; e < 4; e++) {
        x[e] = __fmul_rn(x[e], d.inv_ratio);
        ss += (double) __fmul_rn(x[e], x[e]);
    }
    #pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    const float mean  = (float) (ss / (double) d.idx_dim);
    const float scale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, d.rms_eps)));
    #pragma unroll
    for (int e = 0; e < 4; e++) {
        x[e] = __fmul_rn(x[e], scale);
        if (d.k_norm_w) x[e] = __fmul_rn(x[e], d.k_norm_w[4 * lane + e]);
    }
    // IMRoPE: pair i rotates dims (i, i + rope_dim/2), i < rope_dim/2.  Lane i evaluates pair i's
    // angle (pairs 32.. by further rounds), and every dim of the pair takes it by shuffle.
    const int half = d.rope_dim / 2;
    float y[4] = {x[0], x[1], x[2], x[3]};
    const int sect_dims = d.sections[0] + d.sections[1] + d.sections[2] + d.sections[3];
    const float p = (float) (b * r);
    for (int i0 = 0; i0 < half; i0 += 32) {
        const int i = i0 + lane;                                // this lane's pair
        float c_i = 1.0f, s_i = 0.0f;
        if (i < half) {
            float th = p;
            for (int k = 0; k < i; k++) th = __fmul_rn(th, d.theta_scale);
            const int sector = i % sect_dims;
            const bool use_pos = (sector % 3 == 1 && sector < 3 * d.sections[1]) ||
                                 (sector % 3 == 2 && sector < 3 * d.sections[2]) ||
                                 (sector % 3 == 0 && sector < 3 * d.sections[0]);
            if (!use_pos) th = 0.0f;                            // the 4th section's position is 0
            // cos/sin of the f32 angle (up to ~1e6 rad): Cody-Waite reduction by 2*pi split into two
            // doubles (the product k*2pi_hi is exact to the double rounding of one fma), then
            // sincos of the reduced double argument, rounded once to f32.
            const double td = (double) th;
            const double k = rint(td * 0.15915494309189535);               // 1 / (2 pi)
            double rr = fma(-k, 6.283185307179586, td);                     // 2 pi, high part
            rr = fma(-k, 2.4492935982947064e-16, rr);                       // 2 pi - high part
            double sd, cd;
            sincos(rr, &sd, &cd);
            c_i = (float) cd;
            s_i = (float) sd;
        }
        #pragma unroll
        for (int e = 0; e < 4; e++) {
            const int dim = 4 * lane + e;
            const bool first = dim < half, second = dim >= half && dim < d.rope_dim;
            const int pi = first ? dim : dim - half;                         // pair index of this dim
            const float partner = __shfl_sync(0xffffffffu, x[e], first ? lane + half / 4 : (lane - half / 4) & 31);
            const float c = __shfl_sync(0xffffffffu, c_i, pi & 31), s = __shfl_sync(0xffffffffu, s_i, pi & 31);
            if ((first || second) && pi >= i0 && pi < i0 + 32) {
                if (first) y[e] = __fsub_rn(__fmul_rn(x[e], c), __fmul_rn(partner, s));     // x0*c - x1*s
                else       y[e] = __fadd_rn(__fmul_rn(partner, s), __fmul_rn(x[e], c));     // x0*s + x1*c
            }
        }
    }
    uint2 o;
    o.x = (uint32_t) f32_to_f16_bits(y[0]) | ((uint32_t) f32_to_f16_bits(y[1]) << 16);
    o.y = (uint32_t) f32_to_f16_bits(y[2]) | ((uint32_t) f32_to_f16_bits(y[3]) << 16);
    *reinterpret_cast<uint2 *>(pool_row + 4 * lane) = o;
    if (out_f32) *reinterpret_cast<float4 *>(out_f32 + 4 * lane) = make_float4(y[0], y[1], y[2], y[3]);
}

// ---------------------------------------------------------------------------------------------
// Append of n_tok rows at pos0 (one CTA per token).  Pool updates run afterwards (pool kernel).
__global__ void __launch_bounds__(256) append_rows_kernel(DevDesc d, qsa_layer_cache c, int pos0,
        const float * __restrict__ k, const float * __restrict__ v, const float * __restrict__ kidx) {
    const int t = blockIdx.x, row = pos0 + t;
    c = shard_cache(d, c);
    const int kv_dim = d.n_head_kv * d.head_dim;
    // replicated indexer caches: every row's raw key, only the shard's K/V rows
    const bool kv_here = !d.shard_ri || (row / d.ratio >= d.shard_blk0 && row / d.ratio < d.shard_blk1);
    if (k && kv_here) write_kv_row(d, d.type_k, k + (size_t) t * kv_dim, (uint8_t *) c.k + (size_t) row * d.rb_k, kv_dim);
    if (v && kv_here) write_kv_row(d, d.type_v, v + (size_t) t * kv_dim, (uint8_t *) c.v + (size_t) row * d.rb_v, kv_dim);
    if (kidx)
        for (int i = threadIdx.x; i < d.idx_dim; i += blockDim.x)
            c.idx[(size_t) row * d.idx_dim + i] = f32_to_f16_bits(kidx[(size_t) t * d.idx_dim + i]);
}

// Pooled keys of blocks [blk0, blk0+n_blk): one warp per block.
__global__ void __launch_bounds__(256) pool_blocks_kernel(DevDesc d, const uint16_t * __restrict__ idx,
        uint16_t * __restrict__ pool, int blk0, int n_blk, float * __restrict__ out_f32) {
    pdl_trigger();
    const int j = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (j >= n_blk) return;
    const int64_t b = blk0 + j;
    if (d.shard_blk0 != 0 && !d.shard_ri) {   // a shard's local arrays, indexed by global row / block
        idx = shard_row(idx, (int64_t) d.shard_blk0 * d.ratio, 0, (int64_t) MAX_IDX_DIM * 2);
        pool = shard_row(pool, (int64_t) d.shard_blk0, 0, (int64_t) d.idx_dim * 2);
    }
    pool_block_warp(d, idx + (size_t) b * d.ratio * MAX_IDX_DIM, b, pool + (size_t) b * d.idx_dim,
                    out_f32 ? out_f32 + (size_t) j * d.idx_dim : nullptr);
}

// Decode append for a batch: CTA s (1024 threads) writes row n_past of sequence s (K, V, raw key)
// and, when that row completes its block, the block's pooled key (as the reference recomputes the
// current block every token and stores it, src/qwfn_graph.cpp:470-476; only a complete block's
// pooled key is ever read, an incomplete block being forced by the bias).  The block's raw-key
// rows are staged into shared memory in one round of loads, then summed in order by one warp.
constexpr int APPEND_THREADS = 1024;
// The inputs are plain pointers (no __restrict__): loads through a const __restrict__ pointer may
// be hoisted above the wait.
__global__ void __launch_bounds__(APPEND_THREADS) append_decode_kernel(DevDesc d, const qsa_decode_item * items,
        const float * k, const float * v, const float * kidx, uint32_t * __restrict__ status) {
    extern __shared__ __align__(16) unsigned char dyn_smem[];
    // Launched programmatically behind whatever precedes the call: nothing is read before the
    // kernel ahead has completed (it, in turn, completes only after everything before it).
    pdl_wait();
    pdl_trigger();
    const int s = blockIdx.x;
    qsa_decode_item it = items[s];
    const int row = it.n_past;
    if (row < 0 || row >= d.n_ctx) {
        if (threadIdx.x == 0) set_status(status, DEV_BAD_POS);
        return;
    }
    const bool kv_here = row / d.ratio >= d.shard_blk0 && row / d.ratio < d.shard_blk1;
    if (!kv_here && !d.shard_ri) return;       // another shard's cell
    it.cache = shard_cache(d, it.cache);
    const int kv_dim = d.n_head_kv * d.head_dim;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nb = kv_dim / QK8_0;
    if (!kv_here) {
        // replicated indexer caches: the raw key and pooled key below, K/V on the owning shard
    } else if (d.type_k == QSA_TYPE_Q8_0 && 2 * nb <= (int) (blockDim.x >> 5)) {
        // one q8_0 block per warp: K blocks on warps [0, nb), V blocks on warps [nb, 2 nb)
        if (warp < nb && k)
            quantize_q8_0_warp(k + (size_t) s * kv_dim + warp * QK8_0, (uint8_t *) it.cache.k + (size_t) row * d.rb_k + warp * Q8_0_BYTES, lane);
        else if (warp >= nb && warp < 2 * nb && v)
            quantize_q8_0_warp(v + (size_t) s * kv_dim + (warp - nb) * QK8_0, (uint8_t *) it.cache.v + (size_t) row * d.rb_v + (warp - nb) * Q8_0_BYTES, lane);
    } else {
        if (k) write_kv_row(d, d.type_k, k + (size_t) s * kv_dim, (uint8_t *) it.cache.k + (size_t) row * d.rb_k, kv_dim);
        if (v) write_kv_row(d, d.type_v, v + (size_t) s * kv_dim, (uint8_t *) it.cache.v + (size_t) row * d.rb_v, kv_dim);
    }
    if (kidx) {
        for (int i = threadIdx.x; i < d.idx_dim; i += blockDim.x)
            it.cache.idx[(size_t) row * d.idx_dim + i] = f32_to_f16_bits(kidx[(size_t) s * d.idx_dim + i]);
        if ((row + 1) % d.ratio == 0) {
            __syncthreads();                      // this token's raw key is written
            const int64_t b = row / d.ratio;
            const uint4 * src = reinterpret_cast<const uint4 *>(it.cache.idx + (size_t) b * d.ratio * MAX_IDX_DIM);
            uint4 * rows = reinterpret_cast<uint4 *>(dyn_smem);
            const int n16 = d.ratio * MAX_IDX_DIM / 8;              // 16-byte pieces of the block
            for (int i = threadIdx.x; i < n16; i += blockDim.x) rows[i] = src[i];
            __syncthreads();
            if (threadIdx.x < 32)
                pool_block_warp(d, reinterpret_cast<const uint16_t *>(dyn_smem), b,
                                it.cache.pool + (size_t) b * d.idx_dim, nullptr);
        }
    }
}

}  // namespace qsa
