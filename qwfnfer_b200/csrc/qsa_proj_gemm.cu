// qsa_proj_gemm.cu -- the prefill-sized projections around the node as one tcgen05 GEMM each:
// D[t][n] = sum_k A[t][k] B[n][k], A = the tokens' activations and B = a weight matrix, both
// 16-bit (bf16, or f16 for the q8_0-weight path) and K-major, f32 accumulation in TMEM.
//
// Reference: ggml_mul_mat(W, x) of the attention projections for a prefill chunk
// (src/qwfn_graph.cpp:324-347: attn_q with the gate, attn_k, attn_v, indexer.q_proj, indexer.k_proj)
// and of attn_output (:406-407).
//
// Kernel shape (persistent, one CTA per SM, 192 threads):
//   warp 0   TMA producer: per k-step one 128-row box of A (16 KB) and two 128-row boxes of B
//            (32 KB), 64 columns each with the 128-byte swizzle, into a ring of 4 stages;
//   warp 1   one thread issues 4 tcgen05.mma (kind::f16, M=128, N=256, K=16) per stage into one of
//            two TMEM accumulators (2 x 256 f32 columns), commits each stage back to the producer
//            and each finished tile to the epilogue;
//   warps 2-5  the epilogue, thread = tile row = TMEM lane: reads the 256 columns of its row while
//            the MMAs of the next tile run into the other accumulator.
// Output tile = 128 tokens x 256 weight rows, made of two 128-row halves.  For the projection front
// a tile is one query head, one gate head, one K or V head, or two 128-row indexer halves (query
// heads, then the raw key), and the epilogue applies the head's rms_norm x weight and IMRoPE (the
// arithmetic of qsa_front's decode path) before storing the node's inputs; for attn_output it
// stores the columns as they are.  Every wait is bounded (2 s, DEV_TIMEOUT in the status word).
#include "qsa_kernels.cuh"
#include "qsa_tc.cuh"
#include "qsa_tma.cuh"

namespace qsa {
namespace {

constexpr int PG_BM = 128, PG_BN = 256, PG_BK = 64;
constexpr int PG_STAGES = 4;
constexpr int PG_A_BYTES = PG_BM * PG_BK * 2;                   // 16 KB
constexpr int PG_B_HALF = 128 * PG_BK * 2;                      // 16 KB per 128-row half
constexpr int PG_STAGE_BYTES = PG_A_BYTES + 2 * PG_B_HALF;      // 48 KB
constexpr int PG_THREADS = 192;
constexpr int PG_SMEM = PG_STAGES * PG_STAGE_BYTES + 1024;
constexpr uint32_t PG_TMEM_COLS = 512;                          // two 256-column accumulators

// What an epilogue does with a 128-column half (or a 256-column unit) of a tile.
enum : int { PJ_NONE = 0, PJ_RAW = 1, PJ_NORM_ROPE = 2 };

struct PgMaps {
    CUtensorMap a;          // activations [M][K]
    CUtensorMap b[5];       // weights [rows][K]
};

struct PgArgs {
    int M, K, tiles_m, tiles_n, front;      // front: the projection-front tile map, else plain
    uint32_t idesc;
    // plain: y[t][c] for c < n_cols
    float * y; int ldy, n_cols;
    // front
    int n_head, n_head_kv, idx_n_head, rope_dim;
    float rms_eps;
    const float2 * cs;                      // [M][rope_dim/2] (cos, sin) of each token's rotated pairs
    const float * q_norm; const float * k_norm; const float * q_idx_norm;
    float * q_out; float * gate_out; float * q_idx_out; float * k_out; float * v_out; float * kidx_out;
    uint32_t * status;
};

// Output description of one 128-row half of N tile tn: which B map and rows feed it, and where its
// columns go (unit 256: the two halves are one 256-dim head, normed together).
struct PgHalf {
    int map, row0, mode;
    float * dst; int ld;        // row t of the half's (or unit's) output at dst + t * ld
    const float * w;            // norm weight (null = 1)
};

__device__ __forceinline__ void pg_tile(const PgArgs & a, int tn, PgHalf (&h)[2], bool & unit256) {
    unit256 = false;
    h[0] = PgHalf{-1, 0, PJ_NONE, nullptr, 0, nullptr};
    h[1] = h[0];
    if (!a.front) {                                            // attn_output rows 256 tn ..
        for (int k = 0; k < 2; k++) {
            const int r0 = tn * PG_BN + 128 * k;
            if (r0 < a.n_cols) h[k] = PgHalf{0, r0, PJ_RAW, a.y + r0, a.ldy, nullptr};
        }
        return;
    }
    const int nh = a.n_head, nkv = a.n_head_kv, H = a.idx_n_head;
    if (tn < 2 * nh) {                                         // head tn/2: query rows, then gate rows
        const int hd = tn >> 1, g = tn & 1;
        unit256 = true;
        h[0] = PgHalf{0, (2 * hd + g) * HEAD_DIM, g ? PJ_RAW : PJ_NORM_ROPE,
                      (g ? a.gate_out : a.q_out) + hd * HEAD_DIM, nh * HEAD_DIM, g ? nullptr : a.q_norm};
        h[1] = h[0];
        h[1].row0 += 128;
        return;
    }
    tn -= 2 * nh;
    if (tn < 2 * nkv) {                                        // K heads, then V heads
        const int v = tn >= nkv, g = tn - v * nkv;
        unit256 = true;
        h[0] = PgHalf{1 + v, g * HEAD_DIM, v ? PJ_RAW : PJ_NORM_ROPE, (v ? a.v_out : a.k_out) + g * HEAD_DIM,
                      nkv * HEAD_DIM, v ? nullptr : a.k_norm};
        h[1] = h[0];
        h[1].row0 += 128;
        return;
    }
    tn -= 2 * nkv;
    for (int k = 0; k < 2; k++) {                              // indexer halves: query heads, then the key
        const int j = 2 * tn + k;
        if (j < H) h[k] = PgHalf{3, j * MAX_IDX_DIM, PJ_NORM_ROPE, a.q_idx_out + j * MAX_IDX_DIM, H * MAX_IDX_DIM,
                                 a.q_idx_norm};
        else if (j == H) h[k] = PgHalf{4, 0, PJ_RAW, a.kidx_out, MAX_IDX_DIM, nullptr};
    }
}

__device__ __forceinline__ void pg_ld32(uint32_t taddr, float (&x)[32]) {
    uint32_t v[32];
    tmem_ld32(taddr, v);
    tmem_ld_wait();
    #pragma unroll
    for (int j = 0; j < 32; j++) x[j] = __uint_as_float(v[j]);
}

__device__ __forceinline__ void pg_store32(float * dst, const float (&x)[32]) {
    #pragma unroll
    for (int j = 0; j < 32; j += 4) *reinterpret_cast<float4 *>(dst + j) = make_float4(x[j], x[j + 1], x[j + 2], x[j + 3]);
}

// rms_norm x weight then IMRoPE of one row's D columns (D = 128 or 256) at TMEM address `ta`, stored
// at dst: the arithmetic of qsa_front's norm_rope_warp (f32 squares summed in double, 1/sqrtf in f32,
// pairs (i, i + rope_dim/2) of the first rope_dim columns rotated with the token's (cos, sin)).
// Every lane of the warp runs the TMEM loads (warp-collective); only rows with `valid` store.
__device__ __forceinline__ void pg_norm_rope_row(const PgArgs & a, uint32_t ta, int D, const float * w,
                                                 const float2 * cs, float * dst, bool valid) {
    double ss = 0.0;
    for (int c0 = 0; c0 < D; c0 += 32) {
        float x[32];
        pg_ld32(ta + (uint32_t) c0, x);
        #pragma unroll
        for (int j = 0; j < 32; j++) ss += (double) __fmul_rn(x[j], x[j]);
    }
    const float mean = (float) (ss / (double) D);
    const float scale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, a.rms_eps)));
    const int half = a.rope_dim >> 1;            // a multiple of 32: rope_dim % 64 == 0 (checked on the host)
    for (int c0 = 0; c0 < D; c0 += 32) {
        float x[32];
        pg_ld32(ta + (uint32_t) c0, x);
        #pragma unroll
        for (int j = 0; j < 32; j++) {
            x[j] = __fmul_rn(x[j], scale);
            if (w) x[j] = __fmul_rn(x[j], __ldg(w + c0 + j));
        }
        if (c0 < a.rope_dim) {
            // partner columns: the other half of each rotated pair, normalised the same way
            const int pc0 = c0 < half ? c0 + half : c0 - half;
            float p[32];
            pg_ld32(ta + (uint32_t) pc0, p);
            #pragma unroll
            for (int j = 0; j < 32; j++) {
                p[j] = __fmul_rn(p[j], scale);
                if (w) p[j] = __fmul_rn(p[j], __ldg(w + pc0 + j));
            }
            // the chunk lies wholly inside the rotated columns (rope_dim and half are multiples of 32)
            const bool first = c0 < half;
            const float2 * cc = cs + (first ? c0 : c0 - half);
            #pragma unroll
            for (int j = 0; j < 32; j++) {
                const float2 c = cc[j];
                x[j] = first ? __fsub_rn(__fmul_rn(x[j], c.x), __fmul_rn(p[j], c.y))      // x0*c - x1*s
                             : __fadd_rn(__fmul_rn(p[j], c.y), __fmul_rn(x[j], c.x));     // x0*s + x1*c
            }
        }
        if (valid) pg_store32(dst + c0, x);
    }
}

__global__ void __launch_bounds__(PG_THREADS, 1) proj_gemm_kernel(const __grid_constant__ PgMaps maps, PgArgs a) {
    extern __shared__ __align__(1024) unsigned char pg_smem_raw[];
    __shared__ uint64_t full[PG_STAGES], empty[PG_STAGES], acc_full[2], acc_empty[2], mma_done;
    __shared__ uint32_t tmem_slot;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t raw = smem_u32(pg_smem_raw);
    const uint32_t base = (raw + 1023u) & ~1023u;
    const int n_tiles = a.tiles_m * a.tiles_n;
    const int k_steps = (a.K + PG_BK - 1) / PG_BK;

    if (warp == 0) tmem_alloc_warp(&tmem_slot, PG_TMEM_COLS);
    if (threadIdx.x == 32) {
        for (int s = 0; s < PG_STAGES; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int b = 0; b < 2; b++) {
            mbar_init(&acc_full[b], 1);
            mbar_init(&acc_empty[b], 128);
        }
        mbar_init(&mma_done, 1);
        fence_mbar_init();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tmem_slot;

    if (warp == 0) {
        // ------------------------------------------------------------------ TMA producer
        if (lane == 0) {
            int it = 0;
            bool ok = true;
            for (int tile = blockIdx.x; tile < n_tiles && ok; tile += gridDim.x) {
                const int tm = tile % a.tiles_m, tn = tile / a.tiles_m;
                PgHalf h[2];
                bool unit;
                pg_tile(a, tn, h, unit);
                const uint32_t bytes = PG_A_BYTES + (h[0].map >= 0 ? PG_B_HALF : 0) + (h[1].map >= 0 ? PG_B_HALF : 0);
                for (int ks = 0; ks < k_steps; ks++, it++) {
                    const int s = it % PG_STAGES;
                    if (it >= PG_STAGES && !mbar_poll_bounded(&empty[s], (uint32_t) (((it / PG_STAGES) - 1) & 1), a.status)) {
                        ok = false;
                        break;
                    }
                    const uint32_t sa = base + (uint32_t) (s * PG_STAGE_BYTES);
                    mbar_arrive_expect_tx(&full[s], bytes);
                    tma_load_2d(sa, &maps.a, ks * PG_BK, tm * PG_BM, &full[s]);
                    #pragma unroll
                    for (int k = 0; k < 2; k++)
                        if (h[k].map >= 0)
                            tma_load_2d(sa + PG_A_BYTES + k * PG_B_HALF, &maps.b[h[k].map], ks * PG_BK, h[k].row0, &full[s]);
                }
            }
            // every issued load has landed before the CTA can leave (the most recent phase of each
            // stage used; earlier ones were consumed by the MMA thread)
            for (int j = max(0, it - PG_STAGES); j < it; j++)
                mbar_wait_bounded(&full[j % PG_STAGES], (uint32_t) ((j / PG_STAGES) & 1), a.status);
        }
        __syncwarp();                 // the warp reconverges before the CTA barrier and the TMEM release
    } else if (warp == 1) {
        // ------------------------------------------------------------------ MMA issue (one thread)
        if (lane == 0) {
            int it = 0, tl = 0;
            bool ok = true;
            for (int tile = blockIdx.x; tile < n_tiles && ok; tile += gridDim.x, tl++) {
                const int b = tl & 1;
                if (tl >= 2 && !mbar_wait_bounded(&acc_empty[b], (uint32_t) (((tl >> 1) - 1) & 1), a.status)) break;
                tc_fence_after();
                const uint32_t acc = tmem + (uint32_t) (b * PG_BN);
                for (int ks = 0; ks < k_steps; ks++, it++) {
                    const int s = it % PG_STAGES;
                    if (!mbar_wait_bounded(&full[s], (uint32_t) ((it / PG_STAGES) & 1), a.status)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t sa = base + (uint32_t) (s * PG_STAGE_BYTES), sb = sa + PG_A_BYTES;
                    #pragma unroll
                    for (int kk = 0; kk < PG_BK / 16; kk++)
                        umma_f16(acc, umma_desc_sw128(sa + kk * 32), umma_desc_sw128(sb + kk * 32), a.idesc, ks > 0 || kk > 0);
                    umma_commit(&empty[s]);                  // the stage is free once these MMAs read it
                }
                if (ok) umma_commit(&acc_full[b]);
            }
            umma_commit(&mma_done);                          // every MMA issued above has completed
            mbar_wait_bounded(&mma_done, 0u, a.status);
        }
        __syncwarp();
    } else {
        // ------------------------------------------------------------------ epilogue, thread = row
        const int q = warp & 3, r = q * 32 + lane;
        int tl = 0;
        for (int tile = blockIdx.x; tile < n_tiles; tile += gridDim.x, tl++) {
            const int b = tl & 1;
            const int tm = tile % a.tiles_m, tn = tile / a.tiles_m;
            // one verdict per warp (a lane that saw the phase complete proves it did), so that the
            // warp-collective TMEM loads below never run in part of a warp
            const bool ready = mbar_wait_bounded(&acc_full[b], (uint32_t) ((tl >> 1) & 1), a.status);
            if (!__any_sync(0xffffffffu, ready)) break;
            tc_fence_after();
            PgHalf h[2];
            bool unit;
            pg_tile(a, tn, h, unit);
            // rows past M (a partly filled last row tile) load with the warp but store nothing; the
            // control flow below depends on the tile only, so the warp-collective TMEM loads run in
            // every lane together
            const int t = tm * PG_BM + r;
            const bool valid = t < a.M;
            const uint32_t ta = tmem + ((uint32_t) (q * 32) << 16) + (uint32_t) (b * PG_BN);
            const float2 * cs = a.front ? a.cs + (size_t) (valid ? t : 0) * (a.rope_dim >> 1) : nullptr;
            for (int k = 0; k < (unit ? 1 : 2); k++) {
                const PgHalf & x = h[k];
                const int D = unit ? 256 : 128;
                const uint32_t tk = ta + (uint32_t) (k * 128);
                float * dst = x.dst ? x.dst + (size_t) (valid ? t : 0) * x.ld : nullptr;
                if (x.mode == PJ_NORM_ROPE) {
                    pg_norm_rope_row(a, tk, D, x.w, cs, dst, valid);
                } else if (x.mode == PJ_RAW) {
                    const int ncols = a.front ? D : min(128, a.n_cols - x.row0);
                    for (int c0 = 0; c0 < D; c0 += 32) {
                        float v[32];
                        pg_ld32(tk + (uint32_t) c0, v);
                        if (!valid) continue;
                        if (c0 + 32 <= ncols) {
                            pg_store32(dst + c0, v);
                        } else {
                            for (int j = 0; j < 32 && c0 + j < ncols; j++) dst[c0 + j] = v[j];
                        }
                    }
                }
            }
            tc_fence_before();
            mbar_arrive(&acc_empty[b]);
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc_warp(tmem, PG_TMEM_COLS);
    }
}

// A 16-bit row-major matrix [rows][cols] (cols contiguous, a multiple of 8) as boxes of 64 columns x
// 128 rows with the 128-byte swizzle; out-of-range rows and columns read as zero.
bool encode_rows_map(CUtensorMap * map, const void * ptr, uint64_t rows, uint64_t cols) {
    encode_tiled_fn enc = tensor_map_encoder();
    if (!enc) return false;
    const cuuint64_t dims[2] = {cols, rows};
    const cuuint64_t strides[1] = {cols * 2};
    const cuuint32_t box[2] = {PG_BK, 128};
    const cuuint32_t estr[2] = {1, 1};
    return enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void *>(ptr), dims, strides, box, estr,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

int sm_count() {
    static int n = 0;
    if (!n) {
        int dev = 0;
        if (cudaGetDevice(&dev) != cudaSuccess || cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
            n = 148;
    }
    return n;
}

cudaError_t pg_launch(const PgMaps & maps, PgArgs & a, bool f16, cudaStream_t st) {
    static std::atomic<uint64_t> attr{0};
    cudaError_t e = once_per_device(attr, [] {
        return cudaFuncSetAttribute(proj_gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, PG_SMEM);
    });
    if (e != cudaSuccess) return e;
    a.tiles_m = (a.M + PG_BM - 1) / PG_BM;
    // kind::f16 instruction descriptor: D f32, A and B bf16 (or f16), both K-major, M 128, N 256
    a.idesc = umma_idesc_f16(PG_BM, PG_BN) | (f16 ? 0u : (1u << 7) | (1u << 10));
    const int tiles = a.tiles_m * a.tiles_n;
    const int grid = std::min(tiles, sm_count());
    proj_gemm_kernel<<<grid, PG_THREADS, PG_SMEM, st>>>(maps, a);
    return cudaGetLastError();
}

}  // namespace

int proj_front_tiles(const DevDesc & d) { return 2 * d.n_head + 2 * d.n_head_kv + (d.idx_n_head + 2) / 2; }

cudaError_t launch_proj_gemm_front(const DevDesc & d, cudaStream_t st, int T, int n_embd, const void * xb,
                                   const void * const w[5], bool f16, const float2 * cs, const float * const norm[3],
                                   float * const out[6], uint32_t * status) {
    PgMaps maps;
    const uint64_t rows[5] = {(uint64_t) 2 * HEAD_DIM * d.n_head, (uint64_t) HEAD_DIM * d.n_head_kv,
                              (uint64_t) HEAD_DIM * d.n_head_kv, (uint64_t) MAX_IDX_DIM * d.idx_n_head, MAX_IDX_DIM};
    if (!encode_rows_map(&maps.a, xb, (uint64_t) T, (uint64_t) n_embd)) return cudaErrorNotSupported;
    for (int k = 0; k < 5; k++)
        if (!encode_rows_map(&maps.b[k], w[k], rows[k], (uint64_t) n_embd)) return cudaErrorNotSupported;
    PgArgs a{};
    a.M = T; a.K = n_embd; a.front = 1;
    a.tiles_n = proj_front_tiles(d);
    a.n_head = d.n_head; a.n_head_kv = d.n_head_kv; a.idx_n_head = d.idx_n_head; a.rope_dim = d.rope_dim;
    a.rms_eps = d.rms_eps;
    a.cs = cs;
    a.q_norm = norm[0]; a.k_norm = norm[1]; a.q_idx_norm = norm[2];
    a.q_out = out[0]; a.gate_out = out[1]; a.q_idx_out = out[2]; a.k_out = out[3]; a.v_out = out[4]; a.kidx_out = out[5];
    a.status = status;
    return pg_launch(maps, a, f16, st);
}

cudaError_t launch_proj_gemm_plain(cudaStream_t st, int T, int K, int N, const void * a16, const void * w, bool f16,
                                   float * y, uint32_t * status) {
    PgMaps maps;
    if (!encode_rows_map(&maps.a, a16, (uint64_t) T, (uint64_t) K) || !encode_rows_map(&maps.b[0], w, (uint64_t) N, (uint64_t) K))
        return cudaErrorNotSupported;
    maps.b[1] = maps.b[2] = maps.b[3] = maps.b[4] = maps.b[0];
    PgArgs a{};
    a.M = T; a.K = K; a.front = 0;
    a.tiles_n = (N + PG_BN - 1) / PG_BN;
    a.y = y; a.ldy = N; a.n_cols = N;
    a.status = status;
    return pg_launch(maps, a, f16, st);
}

}  // namespace qsa
