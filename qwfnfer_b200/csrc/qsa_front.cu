// qsa_front.cu -- the projections feeding the sparse-attention node, their norms and IMRoPE.
//
// Reference (graph_builder::sparse_attn_decode, src/qwfn_graph.cpp): indexer.k_proj (:465),
// indexer.q_proj + indexer.q_norm + rope (:479-484), attn_q with query and gate interleaved per
// head + attn_q_norm (:505-510), attn_k + attn_k_norm and attn_v (:512-514), rope of Q and K
// (:515-518); the prefill graph builds the same nodes (:324-347).  ggml_mul_mat over bf16 weights
// converts the f32 activations to bf16 and accumulates the products in f32; rms() is
// ggml_rms_norm over each head followed by the weight multiply (:114-115).
//
// At decode batch sizes this is a matrix-vector product over the layer's projection weights
// (about 48 MB at n_embd 2560): HBM-bound, one pass over the weights per group of 4 tokens.
//   - every CTA owns 32 consecutive rows of one head group (a query+gate head: 512 rows, a K or V
//     head: 256, an indexer query head or the raw indexer key: 128), two CTAs per SM; its 8 warps
//     take 4 rows each and stream the bf16 weights with 16-byte evict-first loads, the next row's
//     loads issued before the current row's products (two rows in flight per warp, ~160 KB per
//     SM); the tokens' activations sit in shared memory as f32 of their bf16 values;
//   - each row's per-token sums (warp-shuffle reduced, a fixed order) go to the workspace; the
//     last CTA of a head group to arrive (an acq_rel counter) normalises the head, applies IMRoPE
//     with the pooled key's angle recurrence, and writes the outputs.
//
// The output side (src/qwfn_graph.cpp:543-545; prefill :406-407): ggml_mul(attn, ggml_sigmoid(gate))
// then ggml_mul_mat(attn_output.weight, .) -- output_kernel: the gated attention output, rounded to
// bf16, in shared memory, and the same weight streaming over attn_output's n_embd rows (16 per CTA).
#include "qsa_kernels.cuh"

namespace qsa {
namespace {

constexpr int FR_THREADS = 256;
constexpr int FR_ROWS    = 32;             // rows per CTA (4 per warp)
constexpr int FR_TOK     = 4;              // tokens per launch
constexpr int FR_UNROLL  = 10;             // 16-byte weight pieces per lane and pass (2560 columns a pass)
constexpr int FR_MAX_EMBD = 12288;          // FR_TOK tokens of activations: 192 KB of shared memory
constexpr int FR_KINDS   = 5;              // query+gate, K, V, indexer query, raw indexer key

struct FrontArgs {
    const uint16_t * w[FR_KINDS];          // bf16 weights of each kind, row-major [rows][n_embd]
    const float * norm[3];                 // q_norm, k_norm, q_idx_norm (may be null)
    const int * pos;                       // [T]
    const float * x;                       // [T][n_embd]
    float * q_out; float * gate_out; float * q_idx_out; float * k_out; float * v_out; float * kidx_out;
    float * y;                             // workspace: [FR_TOK][rows_total]
    unsigned * counters;                   // one per head group
    int n_embd, T, rows_total;
};

struct FrontShape {                        // rows per group, groups and CTAs per group of each kind
    int group_rows[FR_KINDS], groups[FR_KINDS], row0[FR_KINDS], gid0[FR_KINDS];
    int ctas, n_groups;
};

__host__ __device__ inline FrontShape front_shape(const DevDesc & d) {
    FrontShape s;
    const int rows[FR_KINDS] = {2 * HEAD_DIM, HEAD_DIM, HEAD_DIM, MAX_IDX_DIM, MAX_IDX_DIM};
    const int groups[FR_KINDS] = {d.n_head, d.n_head_kv, d.n_head_kv, d.idx_n_head, 1};
    int r = 0, g = 0, c = 0;
    for (int k = 0; k < FR_KINDS; k++) {
        s.group_rows[k] = rows[k];
        s.groups[k] = groups[k];
        s.row0[k] = r;
        s.gid0[k] = g;
        r += rows[k] * groups[k];
        g += groups[k];
        c += groups[k] * (rows[k] / FR_ROWS);
    }
    s.ctas = c;
    s.n_groups = g;
    return s;
}

// cos/sin of the IMRoPE angle of pair i at position `pos`: the pooled key's arithmetic (the angle
// advanced from pos by f32 multiplies by theta_scale, the 4th section at position 0; cos/sin of
// that f32 angle by a reduction by 2*pi split into two doubles and sincos of the reduced double,
// rounded once to f32).
__device__ __forceinline__ float2 rope_cs(const DevDesc & d, float pos, int i) {
    const int sect_dims = d.sections[0] + d.sections[1] + d.sections[2] + d.sections[3];
    float th = pos;
    for (int k = 0; k < i; k++) th = __fmul_rn(th, d.theta_scale);
    const int sector = i % sect_dims;
    const bool use_pos = (sector % 3 == 1 && sector < 3 * d.sections[1]) ||
                         (sector % 3 == 2 && sector < 3 * d.sections[2]) ||
                         (sector % 3 == 0 && sector < 3 * d.sections[0]);
    if (!use_pos) th = 0.0f;
    const double td = (double) th;
    const double k = rint(td * 0.15915494309189535);
    double rr = fma(-k, 6.283185307179586, td);
    rr = fma(-k, 2.4492935982947064e-16, rr);
    double sd, cd;
    sincos(rr, &sd, &cd);
    return make_float2((float) cd, (float) sd);
}

// rms_norm over the warp's D = 32*EPL values (element e of lane l is dim EPL*l + e), times the
// norm weight (the f32 squares summed in double, 1/sqrtf in f32), then IMRoPE with the pair
// table cs[i] = (cos, sin): pair i rotates dims (i, i + rope_dim/2); rope_dim/2 is a multiple of EPL.
template <int EPL>
__device__ __forceinline__ void norm_rope_warp(const DevDesc & d, float (&x)[EPL], const float * __restrict__ w,
                                               const float2 * __restrict__ cs, int lane) {
    constexpr int D = 32 * EPL;
    double ss = 0.0;
    #pragma unroll
    for (int e = 0; e < EPL; e++) ss += (double) __fmul_rn(x[e], x[e]);
    #pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    const float mean  = (float) (ss / (double) D);
    const float scale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, d.rms_eps)));
    #pragma unroll
    for (int e = 0; e < EPL; e++) {
        x[e] = __fmul_rn(x[e], scale);
        if (w) x[e] = __fmul_rn(x[e], w[EPL * lane + e]);
    }
    const int half = d.rope_dim / 2, lane_off = half / EPL;
    float y[EPL];
    #pragma unroll
    for (int e = 0; e < EPL; e++) {
        const int dim = EPL * lane + e;
        const bool first = dim < half, second = dim >= half && dim < d.rope_dim;
        const float partner = __shfl_sync(0xffffffffu, x[e], first ? lane + lane_off : (lane - lane_off) & 31);
        y[e] = x[e];
        if (first || second) {
            const float2 c = cs[first ? dim : dim - half];
            if (first) y[e] = __fsub_rn(__fmul_rn(x[e], c.x), __fmul_rn(partner, c.y));    // x0*c - x1*s
            else       y[e] = __fadd_rn(__fmul_rn(partner, c.y), __fmul_rn(x[e], c.x));    // x0*s + x1*c
        }
    }
    #pragma unroll
    for (int e = 0; e < EPL; e++) x[e] = y[e];
}

__device__ __forceinline__ uint4 ld_stream(const uint4 * p) {
    uint4 v;
    asm volatile("ld.global.cs.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p));
    return v;
}

template <int EPL>
__device__ __forceinline__ void load_head(const float * __restrict__ src, float (&x)[EPL], int lane) {
    #pragma unroll
    for (int e = 0; e < EPL; e += 4) {
        const float4 v = __ldcg(reinterpret_cast<const float4 *>(src + EPL * lane + e));
        x[e] = v.x; x[e + 1] = v.y; x[e + 2] = v.z; x[e + 3] = v.w;
    }
}

template <int EPL>
__device__ __forceinline__ void store_head(float * __restrict__ dst, const float (&x)[EPL], int lane) {
    #pragma unroll
    for (int e = 0; e < EPL; e += 4)
        *reinterpret_cast<float4 *>(dst + EPL * lane + e) = make_float4(x[e], x[e + 1], x[e + 2], x[e + 3]);
}

// One warp's matrix-vector products: rows [0, wrows) of the bf16 matrix at `wrow0` (row stride n
// columns) times the T token vectors in shared memory `xs` ([T][n] f32 of bf16 values).  Work items
// are (row, pass over 32*UNROLL 16-byte pieces of the row); the next item's loads are issued before
// the current item's products, and the first item's loads before `stage_issue` / `stage_wait`
// bring the activations in (every thread of the CTA calls this, and stage_wait ends with the CTA
// barrier).  emit(r, t, sum) is called by lane 0 per finished row r and token t; sums are f32 FMAs
// along each lane's pieces, then a fixed shuffle tree.
template <int UNROLL, typename Issue, typename Wait, typename Emit>
__device__ __forceinline__ void gemv_stream(const uint16_t * __restrict__ wrow0, int wrows, int n, const float * xs, int T,
                                            int lane, Issue && stage_issue, Wait && stage_wait, Emit && emit) {
    const int n16 = n / 8;
    const int passes = (n16 + 32 * UNROLL - 1) / (32 * UNROLL);
    const int items = wrows * passes;
    auto load = [&](int it, uint4 (&v)[UNROLL]) {
        const uint4 * wr = reinterpret_cast<const uint4 *>(wrow0 + (size_t) (it / passes) * n);
        const int base = (it % passes) * 32 * UNROLL + lane;
        #pragma unroll
        for (int u = 0; u < UNROLL; u++) {
            const int i = base + u * 32;
            v[u] = i < n16 ? ld_stream(wr + i) : make_uint4(0u, 0u, 0u, 0u);
        }
    };
    uint4 cur[UNROLL], nxt[UNROLL];
    float acc[FR_TOK];
    #pragma unroll
    for (int t = 0; t < FR_TOK; t++) acc[t] = 0.0f;
    stage_issue();
    if (items > 0) load(0, cur);
    stage_wait();
    for (int it = 0; it < items; it++) {
        if (it + 1 < items) load(it + 1, nxt);
        const int base = (it % passes) * 32 * UNROLL + lane;
        #pragma unroll
        for (int u = 0; u < UNROLL; u++) {
            const int i = base + u * 32;
            if (i >= n16) break;
            const uint32_t p[4] = {cur[u].x, cur[u].y, cur[u].z, cur[u].w};
            float wf[8];
            #pragma unroll
            for (int k = 0; k < 4; k++) {
                wf[2 * k]     = __uint_as_float(p[k] << 16);
                wf[2 * k + 1] = __uint_as_float(p[k] & 0xffff0000u);
            }
            #pragma unroll
            for (int t = 0; t < FR_TOK; t++) {
                if (t >= T) break;
                const float4 x0 = *reinterpret_cast<const float4 *>(xs + (size_t) t * n + 8 * i);
                const float4 x1 = *reinterpret_cast<const float4 *>(xs + (size_t) t * n + 8 * i + 4);
                float s = acc[t];
                s = fmaf(wf[0], x0.x, s); s = fmaf(wf[1], x0.y, s); s = fmaf(wf[2], x0.z, s); s = fmaf(wf[3], x0.w, s);
                s = fmaf(wf[4], x1.x, s); s = fmaf(wf[5], x1.y, s); s = fmaf(wf[6], x1.z, s); s = fmaf(wf[7], x1.w, s);
                acc[t] = s;
            }
        }
        if (it % passes == passes - 1) {                        // the row is complete
            #pragma unroll
            for (int t = 0; t < FR_TOK; t++) {
                float s = acc[t];
                #pragma unroll
                for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
                if (lane == 0 && t < T) emit(it / passes, t, s);
                acc[t] = 0.0f;
            }
        }
        #pragma unroll
        for (int u = 0; u < UNROLL; u++) cur[u] = nxt[u];
    }
}

// The finish of head group g of `kind` for the a.T (<= FR_TOK) tokens of `a`, their projections in
// a.y (row stride a.rows_total): the whole CTA builds the (cos, sin) table of every rotated pair of
// every token; warps 0-3 take token t = warp (norm + IMRoPE, or a copy), warps 4-7 the query
// group's gate half.
__device__ __forceinline__ void front_epilogue(const DevDesc & d, const FrontArgs & a, const FrontShape & sh, int kind,
                                               int g) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, T = a.T;
    // the (cos, sin) of every rotated pair of every token, computed by the whole CTA
    __shared__ float2 cs_tab[FR_TOK][128];
    const int half = d.rope_dim / 2;
    for (int e = tid; e < T * half; e += FR_THREADS)
        cs_tab[e / half][e % half] = rope_cs(d, (float) a.pos[e / half], e % half);
    __syncthreads();
    const int t = warp & 3;                                     // warps 0-3: token t; warps 4-7: token t's gate
    if (t >= T) return;
    const float * yh = a.y + (size_t) t * a.rows_total + sh.row0[kind] + g * sh.group_rows[kind];
    if (kind == 0) {                                            // query (normed, roped) + gate (raw)
        float x[8];
        if (warp < 4) {
            load_head<8>(yh, x, lane);
            norm_rope_warp<8>(d, x, a.norm[0], cs_tab[t], lane);
            store_head<8>(a.q_out + ((size_t) t * d.n_head + g) * HEAD_DIM, x, lane);
        } else {
            load_head<8>(yh + HEAD_DIM, x, lane);
            store_head<8>(a.gate_out + ((size_t) t * d.n_head + g) * HEAD_DIM, x, lane);
        }
    } else if (warp >= 4) {
        return;
    } else if (kind == 1 || kind == 2) {                        // K (normed, roped) or V (raw)
        float x[8];
        load_head<8>(yh, x, lane);
        if (kind == 1) norm_rope_warp<8>(d, x, a.norm[1], cs_tab[t], lane);
        store_head<8>((kind == 1 ? a.k_out : a.v_out) + ((size_t) t * d.n_head_kv + g) * HEAD_DIM, x, lane);
    } else if (kind == 3) {                                     // indexer query (normed, roped)
        float x[4];
        load_head<4>(yh, x, lane);
        norm_rope_warp<4>(d, x, a.norm[2], cs_tab[t], lane);
        store_head<4>(a.q_idx_out + ((size_t) t * d.idx_n_head + g) * MAX_IDX_DIM, x, lane);
    } else {                                                    // raw indexer key
        float x[4];
        load_head<4>(yh, x, lane);
        store_head<4>(a.kidx_out + (size_t) t * MAX_IDX_DIM, x, lane);
    }
}

// Arrival: the last CTA of a head group (of `chunks` CTAs) finishes it.  The barrier orders the
// CTA's row stores before thread 0's release; its acquire orders the other CTAs' stores before our
// reads.
__device__ __forceinline__ void front_finish(const DevDesc & d, const FrontArgs & a, const FrontShape & sh, int kind,
                                             int g, int chunks) {
    __shared__ bool is_last;
    __syncthreads();
    const int gid = sh.gid0[kind] + g;
    if (threadIdx.x == 0) {
        unsigned prev;
        asm volatile("atom.add.acq_rel.gpu.u32 %0, [%1], 1;" : "=r"(prev) : "l"(a.counters + gid) : "memory");
        is_last = prev == (unsigned) chunks - 1;
        if (is_last) a.counters[gid] = 0;                      // leave the counter at zero for the next call
    }
    __syncthreads();
    if (!is_last) return;
    front_epilogue(d, a, sh, kind, g);
}

// This CTA's kind, head group g and 32-row chunk of the group (chunks per group).
__device__ __forceinline__ void front_cta_rows(const FrontShape & sh, int & kind, int & g, int & chunk, int & chunks) {
    int c = blockIdx.x;
    kind = 0;
    while (kind < FR_KINDS - 1 && c >= sh.groups[kind] * (sh.group_rows[kind] / FR_ROWS)) {
        c -= sh.groups[kind] * (sh.group_rows[kind] / FR_ROWS);
        kind++;
    }
    chunks = sh.group_rows[kind] / FR_ROWS;
    g = c / chunks;
    chunk = c % chunks;
}

__global__ void __launch_bounds__(FR_THREADS, 2) front_kernel(DevDesc d, FrontArgs a) {
    extern __shared__ __align__(16) float xs[];                 // [T][n_embd]
    const FrontShape sh = front_shape(d);
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    int kind, g, chunk, chunks;
    front_cta_rows(sh, kind, g, chunk, chunks);
    const int row_in_kind = g * sh.group_rows[kind] + chunk * FR_ROWS;
    const int T = a.T, n = a.n_embd;

    gemv_stream<FR_UNROLL>(a.w[kind] + (size_t) (row_in_kind + warp * (FR_ROWS / 8)) * n, FR_ROWS / 8, n, xs, T, lane,
        [&] {   // the activations go to shared memory by cp.async ahead of the first weight loads' data;
                // each thread then rounds the pieces it copied to bf16 values in place
            for (int i = tid; i < T * n / 4; i += FR_THREADS)
                asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" :: "r"(smem_u32(xs + 4 * i)), "l"(a.x + 4 * i) : "memory");
            asm volatile("cp.async.commit_group;" ::: "memory");
        },
        [&] {
            asm volatile("cp.async.wait_all;" ::: "memory");
            for (int i = tid; i < T * n / 4; i += FR_THREADS) {
                float4 v = reinterpret_cast<float4 *>(xs)[i];
                v.x = __bfloat162float(__float2bfloat16_rn(v.x)); v.y = __bfloat162float(__float2bfloat16_rn(v.y));
                v.z = __bfloat162float(__float2bfloat16_rn(v.z)); v.w = __bfloat162float(__float2bfloat16_rn(v.w));
                reinterpret_cast<float4 *>(xs)[i] = v;
            }
            __syncthreads();
        },
        [&](int r, int t, float v) {
            a.y[(size_t) t * a.rows_total + sh.row0[kind] + row_in_kind + warp * (FR_ROWS / 8) + r] = v;
        });
    front_finish(d, a, sh, kind, g, chunks);
}

constexpr int OUT_ROWS = 16;               // attn_output rows per CTA (2 per warp)
constexpr int OUT_MAX_IN = 4096;           // n_head * head_dim

// y[t][row] = sum_e wo[row][e] * bf16(attn[t][e] * sigmoid(gate[t][e])) for the launch's T tokens; with
// gate null, attn holds the gated product already (f32, or bf16 values when z_bf16).
__global__ void __launch_bounds__(FR_THREADS, 2) output_kernel(const uint16_t * __restrict__ wo, int n_embd, int n_in,
        int T, const float * __restrict__ attn, const float * __restrict__ gate, int z_bf16, float * __restrict__ y) {
    extern __shared__ __align__(16) float zs[];                 // [T][n_in]
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int row0 = blockIdx.x * OUT_ROWS + warp * (OUT_ROWS / 8);
    const int wrows = max(0, min(OUT_ROWS / 8, n_embd - row0));
    gemv_stream<FR_UNROLL>(wo + (size_t) row0 * n_in, wrows, n_in, zs, T, lane,
        [] {},
        [&] {   // ggml_sigmoid: 1 / (1 + exp(-g)) in f32; the product rounded to bf16 as mul_mat converts it
            for (int i = tid; i < T * n_in / 4; i += FR_THREADS) {
                float4 zz;
                if (z_bf16) {
                    const uint2 b = reinterpret_cast<const uint2 *>(attn)[i];
                    zz = make_float4(__uint_as_float(b.x << 16), __uint_as_float(b.x & 0xffff0000u),
                                     __uint_as_float(b.y << 16), __uint_as_float(b.y & 0xffff0000u));
                } else {
                    const float4 o = reinterpret_cast<const float4 *>(attn)[i];
                    const float4 g = gate ? reinterpret_cast<const float4 *>(gate)[i] : make_float4(0.f, 0.f, 0.f, 0.f);
                    auto z = [&](float a, float b) {
                        const float v = gate ? __fmul_rn(a, __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-b)))) : a;
                        return __bfloat162float(__float2bfloat16_rn(v));
                    };
                    zz = make_float4(z(o.x, g.x), z(o.y, g.y), z(o.z, g.z), z(o.w, g.w));
                }
                reinterpret_cast<float4 *>(zs)[i] = zz;
            }
            __syncthreads();
        },
        [&](int r, int t, float v) { y[(size_t) t * n_embd + row0 + r] = v; });
}

// ------------------------------------------------------------------ q8_0 weights
// ggml's mul_mat over q8_0 weights quantises the activation row to q8_0 (its vec_dot_type) and
// takes per 32-value block the integer sum of products times f32(d_w) * f32(d_x), accumulated in
// f32 (ggml_vec_dot_q8_0_q8_0).  Here the activations are quantised with the reference rounding
// (q8_0_quant_lane) and the integer sums are dp4a's.
constexpr int Q8_CHUNK_BLOCKS = 64;                              // q8_0 blocks of a row per streaming step
constexpr int Q8_CHUNK_BYTES  = Q8_CHUNK_BLOCKS * Q8_0_BYTES;    // 2176 bytes, 136 16-byte words
constexpr int Q8_CHUNK_WORDS  = Q8_CHUNK_BYTES / 16;
constexpr int Q8_WPL          = (Q8_CHUNK_WORDS + 31) / 32;      // words a lane loads per step

// Shared memory of a q8_0 GEMV CTA for T tokens of n values: the tokens' q8_0 values and scales,
// then every warp's two weight staging buffers.
inline size_t q8_gemv_smem(int T, int n) {
    return (size_t) T * n + (size_t) T * (n / QK8_0) * 4 + 8 * 2 * Q8_CHUNK_BYTES;
}

// One warp's q8_0 matrix-vector products: rows [0, wrows) of the q8_0 matrix at `wrow0` (rows of
// n/32 blocks of 34 bytes; n a multiple of 256, so a row is a whole number of 16-byte words) times
// the T token rows held as q8_0 in shared memory (xq int8 [T][n], xd f32 [T][n/32]).  A step is one
// row's chunk of up to 64 blocks: the warp loads its 16-byte words (evict-first; the next step's
// loads are issued before this step's products), stages them in one of its two shared buffers, and
// lane = (block of 8, quarter) forms 8 products per token with two dp4a; the block's integer sum is
// reduced over its 4 lanes and times f32(d_w) * f32(d_x) added to the lane's f32 accumulator; at
// the row's end the 8 block slots are summed (fixed shuffle tree) and emit(r, t, sum) is called.
template <typename Emit>
__device__ __forceinline__ void gemv_stream_q8(const uint8_t * __restrict__ wrow0, int wrows, int n, const int8_t * xq,
                                               const float * xd, int T, int lane, uint8_t * wbuf, Emit && emit) {
    const int nb = n / QK8_0;
    const size_t rb = (size_t) nb * Q8_0_BYTES;
    const int chunks = (nb + Q8_CHUNK_BLOCKS - 1) / Q8_CHUNK_BLOCKS;
    const int items = wrows * chunks;
    auto load = [&](int it, uint4 (&v)[Q8_WPL]) {
        const int row = it / chunks, c = it % chunks;
        const int nwords = min(Q8_CHUNK_BLOCKS, nb - c * Q8_CHUNK_BLOCKS) * Q8_0_BYTES / 16;
        const uint4 * p = reinterpret_cast<const uint4 *>(wrow0 + (size_t) row * rb + (size_t) c * Q8_CHUNK_BYTES);
        #pragma unroll
        for (int u = 0; u < Q8_WPL; u++) {
            const int w = lane + 32 * u;
            v[u] = w < nwords ? ld_stream(p + w) : make_uint4(0u, 0u, 0u, 0u);
        }
    };
    uint4 cur[Q8_WPL], nxt[Q8_WPL];
    float acc[FR_TOK];
    #pragma unroll
    for (int t = 0; t < FR_TOK; t++) acc[t] = 0.0f;
    if (items > 0) load(0, cur);
    const int part = lane & 3;
    for (int it = 0; it < items; it++) {
        if (it + 1 < items) load(it + 1, nxt);
        const int c = it % chunks;
        const int nblk = min(Q8_CHUNK_BLOCKS, nb - c * Q8_CHUNK_BLOCKS);     // a multiple of 8
        uint8_t * buf = wbuf + (it & 1) * Q8_CHUNK_BYTES;
        #pragma unroll
        for (int u = 0; u < Q8_WPL; u++) {
            const int w = lane + 32 * u;
            if (w < Q8_CHUNK_WORDS) reinterpret_cast<uint4 *>(buf)[w] = cur[u];
        }
        __syncwarp();
        for (int b = lane >> 2; b < nblk; b += 8) {
            const uint8_t * blk = buf + b * Q8_0_BYTES;
            const float dw = f16_bits_to_f32(*reinterpret_cast<const uint16_t *>(blk));
            const uint32_t w0 = lds_u32_a2(blk + 2 + 8 * part), w1 = lds_u32_a2(blk + 6 + 8 * part);
            const int gb = c * Q8_CHUNK_BLOCKS + b;
            #pragma unroll
            for (int t = 0; t < FR_TOK; t++) {
                if (t >= T) break;
                const uint2 xv = *reinterpret_cast<const uint2 *>(xq + (size_t) t * n + gb * QK8_0 + 8 * part);
                int si = __dp4a((int) w0, (int) xv.x, 0);
                si = __dp4a((int) w1, (int) xv.y, si);
                si += __shfl_xor_sync(0xffffffffu, si, 1);
                si += __shfl_xor_sync(0xffffffffu, si, 2);
                acc[t] = __fadd_rn(acc[t], __fmul_rn((float) si, __fmul_rn(dw, xd[t * nb + gb])));
            }
        }
        if (c == chunks - 1) {                                  // the row is complete
            #pragma unroll
            for (int t = 0; t < FR_TOK; t++) {
                float sacc = acc[t];
                #pragma unroll
                for (int o = 4; o < 32; o <<= 1) sacc += __shfl_xor_sync(0xffffffffu, sacc, o);
                if (lane == 0 && t < T) emit(it / chunks, t, sacc);
                acc[t] = 0.0f;
            }
        }
        #pragma unroll
        for (int u = 0; u < Q8_WPL; u++) cur[u] = nxt[u];
    }
}

// The T token rows (f32, n values each, from global) quantised to q8_0 into shared memory, one
// block per warp in turn; with `gate` each value is first multiplied by sigmoid(gate) (the output
// side's ggml_mul(attn, ggml_sigmoid(gate)) in f32, 1/(1+exp(-g))).
__device__ __forceinline__ void stage_q8(const float * __restrict__ x, const float * __restrict__ gate, int T, int n,
                                         int8_t * xq, float * xd) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nb = n / QK8_0;
    for (int i = warp; i < T * nb; i += FR_THREADS / 32) {
        float v = __ldg(x + (size_t) i * QK8_0 + lane);
        if (gate) v = __fmul_rn(v, __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-__ldg(gate + (size_t) i * QK8_0 + lane)))));
        uint16_t db;
        xq[(size_t) i * QK8_0 + lane] = q8_0_quant_lane(v, db);
        if (lane == 0) xd[i] = f16_bits_to_f32(db);
    }
    __syncthreads();
}

// front_kernel over q8_0 weights (the same rows per CTA, finish and outputs).
__global__ void __launch_bounds__(FR_THREADS, 2) front_kernel_q8(DevDesc d, FrontArgs a) {
    extern __shared__ __align__(16) unsigned char fq_smem[];
    const FrontShape sh = front_shape(d);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    int kind, g, chunk, chunks;
    front_cta_rows(sh, kind, g, chunk, chunks);
    const int T = a.T, n = a.n_embd;
    int8_t * xq = reinterpret_cast<int8_t *>(fq_smem);
    float * xd = reinterpret_cast<float *>(fq_smem + (size_t) T * n);
    uint8_t * wbuf = fq_smem + (size_t) T * n + (size_t) T * (n / QK8_0) * 4 + warp * 2 * Q8_CHUNK_BYTES;
    const int row_in_kind = g * sh.group_rows[kind] + chunk * FR_ROWS;
    const size_t rb = (size_t) (n / QK8_0) * Q8_0_BYTES;
    stage_q8(a.x, nullptr, T, n, xq, xd);
    gemv_stream_q8(reinterpret_cast<const uint8_t *>(a.w[kind]) + (size_t) (row_in_kind + warp * (FR_ROWS / 8)) * rb,
                   FR_ROWS / 8, n, xq, xd, T, lane, wbuf, [&](int r, int t, float v) {
        a.y[(size_t) t * a.rows_total + sh.row0[kind] + row_in_kind + warp * (FR_ROWS / 8) + r] = v;
    });
    front_finish(d, a, sh, kind, g, chunks);
}

// output_kernel over a q8_0 attn_output: z = attn * sigmoid(gate) in f32, quantised to q8_0.
__global__ void __launch_bounds__(FR_THREADS, 2) output_kernel_q8(const uint8_t * __restrict__ wo, int n_embd, int n_in,
        int T, const float * __restrict__ attn, const float * __restrict__ gate, float * __restrict__ y) {
    extern __shared__ __align__(16) unsigned char oq_smem[];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    int8_t * zq = reinterpret_cast<int8_t *>(oq_smem);
    float * zd = reinterpret_cast<float *>(oq_smem + (size_t) T * n_in);
    uint8_t * wbuf = oq_smem + (size_t) T * n_in + (size_t) T * (n_in / QK8_0) * 4 + warp * 2 * Q8_CHUNK_BYTES;
    const int row0 = blockIdx.x * OUT_ROWS + warp * (OUT_ROWS / 8);
    const int wrows = max(0, min(OUT_ROWS / 8, n_embd - row0));
    const size_t rb = (size_t) (n_in / QK8_0) * Q8_0_BYTES;
    stage_q8(attn, gate, T, n_in, zq, zd);
    gemv_stream_q8(wo + (size_t) row0 * rb, wrows, n_in, zq, zd, T, lane, wbuf,
                   [&](int r, int t, float v) { y[(size_t) t * n_embd + row0 + r] = v; });
}

// GEMM-path operands of q8_0 weights: every q8_0 value as f16(f32(d) * q) (a thread per 8 values),
// and activations (f32, optionally times sigmoid(gate)) quantised to q8_0 and stored the same way (a
// warp per block).  The tensor-core products of these f16 values are exact; they differ from the
// integer block sums of the reference only by the f16 rounding of each d * q.
__global__ void q8_to_f16_kernel(const uint8_t * __restrict__ q, uint4 * __restrict__ out, size_t n8) {
    for (size_t i = (size_t) blockIdx.x * blockDim.x + threadIdx.x; i < n8; i += (size_t) gridDim.x * blockDim.x) {
        const uint8_t * blk = q + (i >> 2) * Q8_0_BYTES;
        const float dd = f16_bits_to_f32(*reinterpret_cast<const uint16_t *>(blk));
        const uint8_t * v = blk + 2 + (i & 3) * 8;
        float f[8];
        #pragma unroll
        for (int k = 0; k < 8; k++) f[k] = __fmul_rn(dd, (float) (int8_t) v[k]);
        out[i] = make_uint4(pack_f16x2(f[0], f[1]), pack_f16x2(f[2], f[3]), pack_f16x2(f[4], f[5]), pack_f16x2(f[6], f[7]));
    }
}

__global__ void act_q8_f16_kernel(const float * __restrict__ x, const float * __restrict__ gate, uint16_t * __restrict__ out,
                                  size_t n_blocks) {
    const int lane = threadIdx.x & 31;
    const size_t warps = (size_t) gridDim.x * (blockDim.x / 32);
    for (size_t i = (size_t) blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5); i < n_blocks; i += warps) {
        float v = x[i * QK8_0 + lane];
        if (gate) v = __fmul_rn(v, __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-gate[i * QK8_0 + lane]))));
        uint16_t db;
        const int8_t qv = q8_0_quant_lane(v, db);
        out[i * QK8_0 + lane] = f32_to_f16_bits(__fmul_rn(f16_bits_to_f32(db), (float) qv));
    }
}

constexpr int FR_GEMV_MAX_T = 16;           // above: the projections run as tcgen05 GEMMs (qsa_proj_gemm.cu)

// x (f32) to bf16 (round to nearest even, as the CPU mul_mat converts it), 4 values a thread.
__global__ void to_bf16_kernel(const float4 * __restrict__ x, uint2 * __restrict__ xb, size_t n4) {
    for (size_t i = (size_t) blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += (size_t) gridDim.x * blockDim.x) {
        const float4 v = x[i];
        const uint32_t a0 = __bfloat16_as_ushort(__float2bfloat16_rn(v.x)), a1 = __bfloat16_as_ushort(__float2bfloat16_rn(v.y));
        const uint32_t a2 = __bfloat16_as_ushort(__float2bfloat16_rn(v.z)), a3 = __bfloat16_as_ushort(__float2bfloat16_rn(v.w));
        xb[i] = make_uint2(a0 | (a1 << 16), a2 | (a3 << 16));
    }
}

// z = bf16(attn * sigmoid(gate)) for the output side's GEMM path, 4 values a thread: the arithmetic
// of output_kernel's shared-memory staging.
__global__ void gate_bf16_kernel(const float4 * __restrict__ attn, const float4 * __restrict__ gate,
                                 uint2 * __restrict__ zb, size_t n4) {
    auto z = [](float a, float b) {
        const float sg = __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-b)));
        return (uint32_t) __bfloat16_as_ushort(__float2bfloat16_rn(__fmul_rn(a, sg)));
    };
    for (size_t i = (size_t) blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += (size_t) gridDim.x * blockDim.x) {
        const float4 o = attn[i], g = gate[i];
        zb[i] = make_uint2(z(o.x, g.x) | (z(o.y, g.y) << 16), z(o.z, g.z) | (z(o.w, g.w) << 16));
    }
}

// (cos, sin) of every rotated pair of every token: cs[t][i] = rope_cs(pos[t], i), i < rope_dim/2.
__global__ void rope_table_kernel(DevDesc d, const int * __restrict__ pos, int T, float2 * __restrict__ cs) {
    const int half = d.rope_dim / 2;
    for (int e = blockIdx.x * blockDim.x + threadIdx.x; e < T * half; e += gridDim.x * blockDim.x)
        cs[e] = rope_cs(d, (float) pos[e / half], e % half);
}

// The front's workspace.  Up to FR_GEMV_MAX_T tokens: the status word, the head-group counters and
// FR_TOK tokens' projections.  Above: the status word, the tokens' activations as 16-bit GEMM
// operands (bf16, or f16 of their q8_0 values), their rope table and, for q8_0 weights, the weights
// as f16 GEMM operands.
struct FrontWs { size_t status, counters, y, xb, cs, wdq, total; bool gemm; };

size_t align256(size_t x) { return (x + 255) & ~(size_t) 255; }

// The GEMM path's epilogue rotates 32-column chunks against their partners: rope_dim a multiple of
// 64 (other rope widths run through the GEMV path in token groups).
bool front_gemm_path(const DevDesc & d, int T) { return T > FR_GEMV_MAX_T && d.rope_dim % 64 == 0; }

size_t front_rows(const DevDesc & d) { const FrontShape sh = front_shape(d); return (size_t) sh.row0[FR_KINDS - 1] + MAX_IDX_DIM; }

FrontWs front_ws(const DevDesc & d, int T, int n_embd, int w_type) {
    FrontWs w{};
    w.status = 0;
    w.counters = 16;
    w.gemm = front_gemm_path(d, T);
    if (!w.gemm) {
        w.y = align256(w.counters + (size_t) front_shape(d).n_groups * 4);
        w.total = w.y + (size_t) FR_TOK * front_rows(d) * 4;
    } else {
        w.xb = 256;
        w.cs = align256(w.xb + (size_t) T * n_embd * 2);
        w.wdq = align256(w.cs + (size_t) T * (d.rope_dim / 2) * 8);
        w.total = w_type == QSA_TYPE_Q8_0 ? align256(w.wdq + front_rows(d) * n_embd * 2) : w.wdq;
    }
    return w;
}

unsigned grid_for(size_t n, int per_thread_block = 256) {
    return (unsigned) std::min<size_t>((n + per_thread_block - 1) / per_thread_block, 148 * 8);
}

qsa_status gemm_status(cudaError_t e) {
    return e == cudaSuccess ? QSA_OK : (e == cudaErrorNotSupported ? QSA_ERR_UNSUPPORTED : QSA_ERR_CUDA);
}

// The GEMM path for T > FR_GEMV_MAX_T tokens: the activations as 16-bit operands (bf16; for q8_0
// weights f16 of their q8_0 values, and the weights as f16 of theirs), the rope table, then one
// tcgen05 GEMM over the five weight matrices whose epilogue applies the norms and IMRoPE and stores
// the outputs.
qsa_status front_gemm(const DevDesc & d, const FrontArgs & a, int T, int w_type, const FrontWs & L, unsigned char * wsb,
                      cudaStream_t st) {
    const int n = a.n_embd;
    uint16_t * xb = reinterpret_cast<uint16_t *>(wsb + L.xb);
    float2 * cs = reinterpret_cast<float2 *>(wsb + L.cs);
    const bool q8 = w_type == QSA_TYPE_Q8_0;
    const void * w[5] = {a.w[0], a.w[1], a.w[2], a.w[3], a.w[4]};
    if (q8) {
        const size_t nblk = (size_t) T * n / QK8_0;
        act_q8_f16_kernel<<<grid_for(nblk * 32), 256, 0, st>>>(a.x, nullptr, xb, nblk);
        const FrontShape sh = front_shape(d);
        uint16_t * wdq = reinterpret_cast<uint16_t *>(wsb + L.wdq);
        for (int k = 0; k < FR_KINDS; k++) {
            const size_t rows = (size_t) sh.groups[k] * sh.group_rows[k];
            uint16_t * dst = wdq + (size_t) sh.row0[k] * n;
            q8_to_f16_kernel<<<grid_for(rows * n / 8), 256, 0, st>>>(static_cast<const uint8_t *>(w[k]),
                                                                    reinterpret_cast<uint4 *>(dst), rows * n / 8);
            w[k] = dst;
        }
    } else {
        const size_t n4 = (size_t) T * n / 4;
        to_bf16_kernel<<<grid_for(n4), 256, 0, st>>>(reinterpret_cast<const float4 *>(a.x), reinterpret_cast<uint2 *>(xb), n4);
    }
    rope_table_kernel<<<grid_for((size_t) T * (d.rope_dim / 2)), 256, 0, st>>>(d, a.pos, T, cs);
    if (cudaGetLastError() != cudaSuccess) return QSA_ERR_CUDA;
    const float * norm[3] = {a.norm[0], a.norm[1], a.norm[2]};
    float * out[6] = {a.q_out, a.gate_out, a.q_idx_out, a.k_out, a.v_out, a.kidx_out};
    return gemm_status(launch_proj_gemm_front(d, st, T, n, xb, w, q8, cs, norm, out,
                                              reinterpret_cast<uint32_t *>(wsb + L.status)));
}

bool aligned16(const void * p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Weight formats of the projections: bf16 rows (n a multiple of 8), or q8_0 rows (n a multiple of
// 256: whole 16-byte words per row, and whole 8-block groups for the GEMV's lane layout).
bool weight_shape_ok(int w_type, int n) {
    if (w_type == QSA_TYPE_BF16) return n % 8 == 0;
    if (w_type == QSA_TYPE_Q8_0) return n % 256 == 0;
    return false;
}

}  // namespace
}  // namespace qsa

using namespace qsa;

extern "C" size_t qsa_front_workspace_size(const qsa_desc * dd, const qsa_front_weights * w, int32_t T) {
    if (qsa_desc_check(dd) != QSA_OK || !w || T <= 0 || w->n_embd <= 0) return 0;
    return front_ws(dev_desc(dd), T, w->n_embd, w->w_type).total;
}

extern "C" qsa_status qsa_front(const qsa_desc * dd, const qsa_front_weights * w, int32_t T, const int32_t * pos,
                                const float * x, float * q_out, float * gate_out, float * q_idx_out,
                                float * k_out, float * v_out, float * kidx_out,
                                void * ws, size_t ws_bytes, qsa_stream_t stream) {
    qsa_status s = qsa_desc_check(dd);
    if (s != QSA_OK) return s;
    if (!w || T <= 0 || !pos || !x || !q_out || !gate_out || !q_idx_out || !k_out || !v_out || !kidx_out)
        return QSA_ERR_INVALID;
    if (!w->wq || !w->wk || !w->wv || !w->wq_idx || !w->wk_idx) return QSA_ERR_INVALID;
    if (w->w_type != QSA_TYPE_BF16 && w->w_type != QSA_TYPE_Q8_0) return QSA_ERR_UNSUPPORTED;
    if (w->n_embd <= 0 || !weight_shape_ok(w->w_type, w->n_embd) || w->n_embd > FR_MAX_EMBD) return QSA_ERR_UNSUPPORTED;
    if (dd->rope_dim % 16 != 0) return QSA_ERR_UNSUPPORTED;          // pairs at a lane distance for 8 values a lane
    const void * ptrs[] = {w->wq, w->wk, w->wv, w->wq_idx, w->wk_idx, x, q_out, gate_out, q_idx_out, k_out, v_out, kidx_out};
    for (const void * p : ptrs)
        if (!aligned16(p)) return QSA_ERR_INVALID;
    const bool q8 = w->w_type == QSA_TYPE_Q8_0;
    const DevDesc d = dev_desc(dd);
    const FrontWs L = front_ws(d, T, w->n_embd, w->w_type);
    if (!ws || ws_bytes < L.total) return QSA_ERR_WORKSPACE;
    // the GEMM path's tensor maps want their base addresses 16-byte aligned (slices of ws at 256)
    if (L.gemm && !aligned16(ws)) return QSA_ERR_WORKSPACE;
    static std::atomic<uint64_t> attr{0};
    cudaError_t e = once_per_device(attr, [] {
        cudaError_t r = cudaFuncSetAttribute(front_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, FR_TOK * FR_MAX_EMBD * 4);
        if (r == cudaSuccess)
            r = cudaFuncSetAttribute(front_kernel_q8, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     (int) q8_gemv_smem(FR_TOK, FR_MAX_EMBD));
        return r;
    });
    if (e != cudaSuccess) return QSA_ERR_CUDA;
    const FrontShape sh = front_shape(d);
    unsigned char * wsb = static_cast<unsigned char *>(ws);
    FrontArgs a{};
    a.w[0] = static_cast<const uint16_t *>(w->wq);
    a.w[1] = static_cast<const uint16_t *>(w->wk);
    a.w[2] = static_cast<const uint16_t *>(w->wv);
    a.w[3] = static_cast<const uint16_t *>(w->wq_idx);
    a.w[4] = static_cast<const uint16_t *>(w->wk_idx);
    a.norm[0] = w->q_norm; a.norm[1] = w->k_norm; a.norm[2] = w->q_idx_norm;
    a.counters = reinterpret_cast<unsigned *>(wsb + L.counters);
    a.y = reinterpret_cast<float *>(wsb + L.y);
    a.n_embd = w->n_embd;
    a.rows_total = (int) front_rows(d);
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    if (L.gemm) {
        a.pos = pos; a.x = x; a.q_out = q_out; a.gate_out = gate_out; a.q_idx_out = q_idx_out;
        a.k_out = k_out; a.v_out = v_out; a.kidx_out = kidx_out;
        return front_gemm(d, a, T, w->w_type, L, wsb, st);
    }
    const size_t kv = (size_t) d.n_head_kv * HEAD_DIM;
    for (int t0 = 0; t0 < T; t0 += FR_TOK) {                   // token groups run one after another on the stream
        a.T = std::min(FR_TOK, T - t0);
        a.pos = pos + t0;
        a.x = x + (size_t) t0 * w->n_embd;
        a.q_out = q_out + (size_t) t0 * d.n_head * HEAD_DIM;
        a.gate_out = gate_out + (size_t) t0 * d.n_head * HEAD_DIM;
        a.q_idx_out = q_idx_out + (size_t) t0 * d.idx_n_head * MAX_IDX_DIM;
        a.k_out = k_out + t0 * kv;
        a.v_out = v_out + t0 * kv;
        a.kidx_out = kidx_out + (size_t) t0 * MAX_IDX_DIM;
        if (q8) front_kernel_q8<<<sh.ctas, FR_THREADS, q8_gemv_smem(a.T, w->n_embd), st>>>(d, a);
        else    front_kernel<<<sh.ctas, FR_THREADS, (size_t) a.T * w->n_embd * 4, st>>>(d, a);
        if ((e = cudaGetLastError()) != cudaSuccess) return QSA_ERR_CUDA;
    }
    return QSA_OK;
}

// The output side's workspace: none up to FR_GEMV_MAX_T tokens; above, the status word, the gated
// activations as the GEMM's 16-bit A operand (bf16, or f16 of their q8_0 values for q8_0 weights)
// and, for q8_0 weights, attn_output as f16.
size_t out_ws_bytes(const qsa_desc * d, int n_embd, int T, int w_type, size_t * z_off, size_t * w_off) {
    if (T <= FR_GEMV_MAX_T) return 0;
    const size_t n_in = (size_t) d->n_head * d->head_dim;
    *z_off = 256;
    *w_off = align256(*z_off + (size_t) T * n_in * 2);
    return w_type == QSA_TYPE_Q8_0 ? align256(*w_off + (size_t) n_embd * n_in * 2) : *w_off;
}

extern "C" size_t qsa_output_workspace_size(const qsa_desc * dd, int32_t n_embd, int32_t w_type, int32_t T) {
    if (qsa_desc_check(dd) != QSA_OK || n_embd <= 0 || T <= 0) return 0;
    if (w_type != QSA_TYPE_BF16 && w_type != QSA_TYPE_Q8_0) return 0;
    size_t a = 0, b = 0;
    return out_ws_bytes(dd, n_embd, T, w_type, &a, &b);
}

extern "C" qsa_status qsa_output(const qsa_desc * dd, const void * wo, int32_t n_embd, int32_t w_type, int32_t T,
                                 const float * attn, const float * gate, float * y, void * ws, size_t ws_bytes,
                                 qsa_stream_t stream) {
    qsa_status s = qsa_desc_check(dd);
    if (s != QSA_OK) return s;
    if (!wo || !attn || !gate || !y || T <= 0 || n_embd <= 0) return QSA_ERR_INVALID;
    if (w_type != QSA_TYPE_BF16 && w_type != QSA_TYPE_Q8_0) return QSA_ERR_UNSUPPORTED;
    if (!aligned16(wo) || !aligned16(attn) || !aligned16(gate) || (reinterpret_cast<uintptr_t>(y) & 3u))
        return QSA_ERR_INVALID;
    const int n_in = dd->n_head * dd->head_dim;
    if (n_in > OUT_MAX_IN || !weight_shape_ok(w_type, n_in)) return QSA_ERR_UNSUPPORTED;
    const bool q8 = w_type == QSA_TYPE_Q8_0;
    size_t z_off = 0, w_off = 0;
    const size_t need = out_ws_bytes(dd, n_embd, T, w_type, &z_off, &w_off);
    if (need && (!ws || ws_bytes < need || !aligned16(ws))) return QSA_ERR_WORKSPACE;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    if (T > FR_GEMV_MAX_T) {       // a prefill-sized batch: y = z wo^T as one GEMM
        if (n_embd % 4 != 0) return QSA_ERR_UNSUPPORTED;      // float4 rows of the epilogue's stores
        if (!aligned16(y)) return QSA_ERR_INVALID;
        unsigned char * wsb = static_cast<unsigned char *>(ws);
        uint16_t * zb = reinterpret_cast<uint16_t *>(wsb + z_off);
        const void * w16 = wo;
        if (q8) {
            const size_t nblk = (size_t) T * n_in / QK8_0;
            act_q8_f16_kernel<<<grid_for(nblk * 32), 256, 0, st>>>(attn, gate, zb, nblk);
            uint16_t * wdq = reinterpret_cast<uint16_t *>(wsb + w_off);
            const size_t n8 = (size_t) n_embd * n_in / 8;
            q8_to_f16_kernel<<<grid_for(n8), 256, 0, st>>>(static_cast<const uint8_t *>(wo), reinterpret_cast<uint4 *>(wdq), n8);
            w16 = wdq;
        } else {
            const size_t n4 = (size_t) T * n_in / 4;
            gate_bf16_kernel<<<grid_for(n4), 256, 0, st>>>(reinterpret_cast<const float4 *>(attn),
                                                          reinterpret_cast<const float4 *>(gate), reinterpret_cast<uint2 *>(zb), n4);
        }
        if (cudaGetLastError() != cudaSuccess) return QSA_ERR_CUDA;
        return gemm_status(launch_proj_gemm_plain(st, T, n_in, n_embd, zb, w16, q8, y, reinterpret_cast<uint32_t *>(wsb)));
    }
    static std::atomic<uint64_t> attr{0};
    cudaError_t e = once_per_device(attr, [] {
        cudaError_t r = cudaFuncSetAttribute(output_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, FR_TOK * OUT_MAX_IN * 4);
        if (r == cudaSuccess)
            r = cudaFuncSetAttribute(output_kernel_q8, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     (int) q8_gemv_smem(FR_TOK, OUT_MAX_IN));
        return r;
    });
    if (e != cudaSuccess) return QSA_ERR_CUDA;
    const unsigned grid = (unsigned) ((n_embd + OUT_ROWS - 1) / OUT_ROWS);
    for (int t0 = 0; t0 < T; t0 += FR_TOK) {
        const int Tg = std::min(FR_TOK, T - t0);
        if (q8)
            output_kernel_q8<<<grid, FR_THREADS, q8_gemv_smem(Tg, n_in), st>>>(
                static_cast<const uint8_t *>(wo), n_embd, n_in, Tg, attn + (size_t) t0 * n_in, gate + (size_t) t0 * n_in,
                y + (size_t) t0 * n_embd);
        else
            output_kernel<<<grid, FR_THREADS, (size_t) Tg * n_in * 4, st>>>(
                static_cast<const uint16_t *>(wo), n_embd, n_in, Tg, attn + (size_t) t0 * n_in, gate + (size_t) t0 * n_in,
                0, y + (size_t) t0 * n_embd);
        if ((e = cudaGetLastError()) != cudaSuccess) return QSA_ERR_CUDA;
    }
    return QSA_OK;
}

// The output projection over the gated product the attention already wrote (qsa_decode_gated /
// qsa_prefill_gated): z bf16 (bf16 weights) or f32 (either weight type) [T][n_head*head_dim].
extern "C" qsa_status qsa_output_z(const qsa_desc * dd, const void * wo, int32_t n_embd, int32_t w_type, int32_t T,
                                   const void * z, int32_t z_type, float * y, void * ws, size_t ws_bytes,
                                   qsa_stream_t stream) {
    qsa_status s = qsa_desc_check(dd);
    if (s != QSA_OK) return s;
    if (!wo || !z || !y || T <= 0 || n_embd <= 0) return QSA_ERR_INVALID;
    if (w_type != QSA_TYPE_BF16 && w_type != QSA_TYPE_Q8_0) return QSA_ERR_UNSUPPORTED;
    if (z_type != QSA_TYPE_F32 && !(z_type == QSA_TYPE_BF16 && w_type == QSA_TYPE_BF16)) return QSA_ERR_INVALID;
    if (!aligned16(wo) || !aligned16(z) || (reinterpret_cast<uintptr_t>(y) & 3u)) return QSA_ERR_INVALID;
    const int n_in = dd->n_head * dd->head_dim;
    if (n_in > OUT_MAX_IN || !weight_shape_ok(w_type, n_in)) return QSA_ERR_UNSUPPORTED;
    const bool q8 = w_type == QSA_TYPE_Q8_0, zb16 = z_type == QSA_TYPE_BF16;
    size_t z_off = 0, w_off = 0;
    const size_t need = out_ws_bytes(dd, n_embd, T, w_type, &z_off, &w_off);
    if (need && (!ws || ws_bytes < need || !aligned16(ws))) return QSA_ERR_WORKSPACE;
    cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
    if (T > FR_GEMV_MAX_T) {
        if (n_embd % 4 != 0) return QSA_ERR_UNSUPPORTED;
        if (!aligned16(y)) return QSA_ERR_INVALID;
        unsigned char * wsb = static_cast<unsigned char *>(ws);
        const void * a16 = z;                  // bf16 z enters the GEMM as it is
        const void * w16 = wo;
        if (!zb16) {
            uint16_t * zb = reinterpret_cast<uint16_t *>(wsb + z_off);
            if (q8) {
                const size_t nblk = (size_t) T * n_in / QK8_0;
                act_q8_f16_kernel<<<grid_for(nblk * 32), 256, 0, st>>>(static_cast<const float *>(z), nullptr, zb, nblk);
            } else {
                const size_t n4 = (size_t) T * n_in / 4;
                to_bf16_kernel<<<grid_for(n4), 256, 0, st>>>(static_cast<const float4 *>(z), reinterpret_cast<uint2 *>(zb), n4);
            }
            a16 = zb;
        }
        if (q8) {
            uint16_t * wdq = reinterpret_cast<uint16_t *>(wsb + w_off);
            const size_t n8 = (size_t) n_embd * n_in / 8;
            q8_to_f16_kernel<<<grid_for(n8), 256, 0, st>>>(static_cast<const uint8_t *>(wo), reinterpret_cast<uint4 *>(wdq), n8);
            w16 = wdq;
        }
        if (cudaGetLastError() != cudaSuccess) return QSA_ERR_CUDA;
        return gemm_status(launch_proj_gemm_plain(st, T, n_in, n_embd, a16, w16, q8, y, reinterpret_cast<uint32_t *>(wsb)));
    }
    static std::atomic<uint64_t> attr{0};
    cudaError_t e = once_per_device(attr, [] {
        cudaError_t r = cudaFuncSetAttribute(output_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, FR_TOK * OUT_MAX_IN * 4);
        if (r == cudaSuccess)
            r = cudaFuncSetAttribute(output_kernel_q8, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     (int) q8_gemv_smem(FR_TOK, OUT_MAX_IN));
        return r;
    });
    if (e != cudaSuccess) return QSA_ERR_CUDA;
    const unsigned grid = (unsigned) ((n_embd + OUT_ROWS - 1) / OUT_ROWS);
    const size_t zes = zb16 ? 2 : 4;
    for (int t0 = 0; t0 < T; t0 += FR_TOK) {
        const int Tg = std::min(FR_TOK, T - t0);
        const float * zt = reinterpret_cast<const float *>(static_cast<const unsigned char *>(z) + (size_t) t0 * n_in * zes);
        if (q8)
            output_kernel_q8<<<grid, FR_THREADS, q8_gemv_smem(Tg, n_in), st>>>(
                static_cast<const uint8_t *>(wo), n_embd, n_in, Tg, zt, nullptr, y + (size_t) t0 * n_embd);
        else
            output_kernel<<<grid, FR_THREADS, (size_t) Tg * n_in * 4, st>>>(
                static_cast<const uint16_t *>(wo), n_embd, n_in, Tg, zt, nullptr, zb16 ? 1 : 0, y + (size_t) t0 * n_embd);
        if ((e = cudaGetLastError()) != cudaSuccess) return QSA_ERR_CUDA;
    }
    return QSA_OK;
}
