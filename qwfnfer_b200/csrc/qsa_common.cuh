// qsa_common.cuh -- shared device-side definitions of libqsa (sm_100a).
#pragma once

#include <cstdint>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "../../include/qsa.h"

namespace qsa {

constexpr int QK8_0        = 32;   // q8_0 block: { f16 d; int8 qs[32] }
constexpr int Q8_0_BYTES   = 34;
constexpr int HEAD_DIM     = 256;  // the attention kernels are written for head_dim 256
constexpr int GQA_TILE     = 8;    // query heads per KV head packed into one MMA N tile
constexpr int CELLS_TILE   = 64;   // cells per pipeline stage of the attention kernel
constexpr int MAX_IDX_DIM  = 128;  // indexer key length handled by the pooling/scoring kernels

// Status word codes written by kernels (the host maps them onto qsa_status).
enum : uint32_t { DEV_OK = 0, DEV_BAD_POS = 1u << 0, DEV_TIMEOUT = 1u << 1, DEV_BAD_SEL = 1u << 2 };

// Descriptor as the kernels see it: the public qsa_desc plus values derived on the host.
struct DevDesc {
    int n_head, n_head_kv, head_dim, gqa;
    int idx_n_head, idx_dim, ratio, top_k, n_force, kb, window;
    int n_ctx, type_k, type_v, rope_dim;
    int sections[4];
    float rms_eps;
    float theta_scale;      // powf(rope_freq_base, -2/rope_dim), computed by the host libm
    float inv_ratio;        // 1.0f / ratio
    float scale_log2;       // log2(e) / sqrt(head_dim)
    const float * k_norm_w; // may be null
    int64_t rb_k, rb_v;     // bytes per K/V cache row (all heads)
    int hb_k, hb_v;         // bytes of one head inside a row
    // KV-sequence sharding: this device holds blocks [shard_blk0, shard_blk1) of every cache, in
    // local arrays whose row 0 is cell shard_blk0 * ratio (pooled row 0 is block shard_blk0).
    // Unsharded: [0, INT_MAX).
    int shard_blk0, shard_blk1;
    // Replicated indexer caches: with shard_ri set only K and V are local to the shard; the raw
    // keys and pooled keys of every block are held (global rows) and every rank selects globally.
    int shard_ri;
    // K and V in pinned host memory (qsa_desc.placement & QSA_KV_HOST): read with ordinary loads,
    // never by bulk or tensor copies.
    int kv_host;
};

// Local address of global row `row` of a sharded cache array with `row_bytes` per row; rows
// before the shard are never dereferenced (the callers stay inside [shard_blk0, shard_blk1)).
template <typename T>
__device__ __forceinline__ T * shard_row(T * base, int64_t row0, int64_t row, int64_t row_bytes) {
    return reinterpret_cast<T *>(reinterpret_cast<uintptr_t>(base) + (uintptr_t) ((row - row0) * row_bytes));
}

// A shard's cache arrays re-based so that global rows index them (identity when unsharded).
__device__ __forceinline__ qsa_layer_cache shard_cache(const DevDesc & d, qsa_layer_cache c) {
    if (d.shard_blk0 != 0) {
        const int64_t row0 = (int64_t) d.shard_blk0 * d.ratio;
        c.k = shard_row(c.k, row0, 0, d.rb_k);
        c.v = shard_row(c.v, row0, 0, d.rb_v);
        if (!d.shard_ri) {
            c.idx = shard_row(c.idx, row0, 0, (int64_t) d.idx_dim * 2);
            c.pool = shard_row(c.pool, (int64_t) d.shard_blk0, 0, (int64_t) d.idx_dim * 2);
        }
    }
    return c;
}

// ------------------------------------------------------------------ small helpers
__device__ __forceinline__ float f16_bits_to_f32(uint16_t u) { return __half2float(__ushort_as_half(u)); }
__device__ __forceinline__ uint16_t f32_to_f16_bits(float f) { return __half_as_ushort(__float2half_rn(f)); }

__device__ __forceinline__ float warp_max(float v) {
    #pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}
__device__ __forceinline__ double warp_sum16_d(double v) {   // butterfly within aligned 16-lane halves
    #pragma unroll
    for (int o = 8; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// One q8_0 block (32 values) across a warp, lane = element, with ggml's reference rounding
// (quantize_row_q8_0_ref): d = amax/127, id = 1/d (0 when d == 0), q = roundf(x*id), d stored as
// f16.  Returns the lane's quantised value; dbits receives the f16 bits of d (in every lane).
__device__ __forceinline__ int8_t q8_0_quant_lane(float v, uint16_t & dbits) {
    float amax = fabsf(v);
    #pragma unroll
    for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    const float d  = __fdiv_rn(amax, 127.0f);
    const float id = d != 0.0f ? __fdiv_rn(1.0f, d) : 0.0f;
    dbits = f32_to_f16_bits(d);
    return (int8_t) (int) roundf(__fmul_rn(v, id));
}

// Programmatic dependent launch: a kernel launched with programmatic stream serialization may
// start while its predecessor runs; it must wait before touching what the predecessor writes.
// Triggering lets the successor launch once every CTA of this grid has started or exited.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// Loads of data that the preceding grid of a programmatic chain writes, issued after pdl_wait():
// volatile asm with a memory clobber is never moved above the wait (through a const __restrict__
// pointer the compiler may treat the data as unchanging for the whole kernel and hoist its loads),
// and .cg reads the lines from L2.
__device__ __forceinline__ int ld_dep(const int * p) {
    int v;
    asm volatile("ld.global.cg.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ float ld_dep(const float * p) {
    float v;
    asm volatile("ld.global.cg.f32 %0, [%1];" : "=f"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ float4 ld_dep(const float4 * p) {
    float4 v;
    asm volatile("ld.global.cg.v4.f32 {%0,%1,%2,%3}, [%4];" : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ uint4 ld_dep(const uint4 * p) {
    uint4 v;
    asm volatile("ld.global.cg.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ void set_status(uint32_t * status, uint32_t code) {
    if (status) atomicOr(status, code);
}

// ------------------------------------------------------------------ the node's output
// Where the attention output goes: `out` (f32 [n_q][n_head][head_dim], optional) and, with a gate,
// the gated product z = out * sigmoid(gate) of the node's output side (ggml_mul(attn,
// ggml_sigmoid(gate)), f32, sigmoid 1/(1+exp(-g))), stored as bf16 (rounded as the bf16
// attn_output mul_mat converts it) or as f32 (z_bf16 = 0); gate and z are [n_q][n_head*head_dim].
struct OutSpec {
    float * out;
    const float * gate;
    void * z;
    int z_bf16;
};

// Where a sharded decode's unnormalised states go: query t's state at base[p] + t x the state
// floats, for every p < n (n = 0: no state, the output instead; n = 1: this rank's workspace; with
// the NVLink peer exchange, this rank's slot in every rank's gather region, remote ones included).
// The writers do not fence: the kernel that publishes the states waits for the writing grid to
// complete (griddepcontrol.wait: its stores performed and visible to the waiting thread), and its
// system-scope release of the flag carries them to the peers.  A fence in every writing thread
// waited for its own NVLink acknowledgements and lengthened the merge from 24 to 42 us (batched).
constexpr int MAX_STATE_DST = 8;
struct StateDst {
    float * base[MAX_STATE_DST];
    int n;
};
// (unrolled over the fixed slots: a runtime index into the kernel parameter would copy it to the
// stack)
__device__ __forceinline__ void state_put4(const StateDst & s, size_t off, float4 v) {
    #pragma unroll
    for (int p = 0; p < MAX_STATE_DST; p++)
        if (p < s.n) *reinterpret_cast<float4 *>(s.base[p] + off) = v;
}
__device__ __forceinline__ void state_put(const StateDst & s, size_t off, float v) {
    #pragma unroll
    for (int p = 0; p < MAX_STATE_DST; p++)
        if (p < s.n) s.base[p][off] = v;
}

// Four consecutive output values at element offset `off` (a multiple of 4).
__device__ __forceinline__ void out_store4(const OutSpec & o, size_t off, float4 v) {
    if (o.out) *reinterpret_cast<float4 *>(o.out + off) = v;
    if (o.z) {
        const float4 g = *reinterpret_cast<const float4 *>(o.gate + off);
        auto gz = [](float a, float b) { return __fmul_rn(a, __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-b)))); };
        const float z0 = gz(v.x, g.x), z1 = gz(v.y, g.y), z2 = gz(v.z, g.z), z3 = gz(v.w, g.w);
        if (o.z_bf16) {
            auto b16 = [](float x) { return (uint32_t) __bfloat16_as_ushort(__float2bfloat16_rn(x)); };
            *reinterpret_cast<uint2 *>(static_cast<uint16_t *>(o.z) + off) = make_uint2(b16(z0) | (b16(z1) << 16),
                                                                                        b16(z2) | (b16(z3) << 16));
        } else {
            *reinterpret_cast<float4 *>(static_cast<float *>(o.z) + off) = make_float4(z0, z1, z2, z3);
        }
    }
}

// ------------------------------------------------------------------ mbarrier + bulk copy
__device__ __forceinline__ uint32_t smem_u32(const void * p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint64_t * bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" :: "r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t * bar) {
    asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];" :: "r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t * bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 _, [%0], %1;"
                 :: "r"(smem_u32(bar)), "r"(bytes) : "memory");
}
// One probe of the phase; returns true when the phase with `parity` has completed.  A thread
// whose phase is still open is suspended in hardware until it completes or about 20 us pass (the
// time hint), so waiting costs few instructions.
__device__ __forceinline__ bool mbar_try_wait(uint64_t * bar, uint32_t parity) {
    uint32_t done;
    asm volatile("{\n\t.reg .pred p;\n\t"
                 "mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2, %3;\n\t"
                 "selp.u32 %0, 1, 0, p;\n\t}"
                 : "=r"(done) : "r"(smem_u32(bar)), "r"(parity), "r"(20000u) : "memory");
    return done != 0;
}
__device__ __forceinline__ uint64_t global_timer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
// Wait at most ~2 s of wall time; on running out, flag DEV_TIMEOUT and return false (the
// caller then skips its work; the host sees QSA_ERR_TIMEOUT from qsa_check).
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t * bar, uint32_t parity, uint32_t * status) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = global_timer_ns();
    for (;;) {
        if (mbar_try_wait(bar, parity)) return true;
        if (global_timer_ns() - t0 > 2000000000ull) break;
    }
    set_status(status, DEV_TIMEOUT);
    return false;
}
// Non-tensor bulk copy global -> this CTA's shared memory, completing on `bar`.
// Both addresses 16-byte aligned, bytes a multiple of 16; the destination is this CTA only.
__device__ __forceinline__ void bulk_g2s(void * dst, const void * src, uint32_t bytes, uint64_t * bar) {
    asm volatile("cp.async.bulk.shared::cta.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
                 :: "r"(smem_u32(dst)), "l"(src), "r"(bytes), "r"(smem_u32(bar)) : "memory");
}

// ------------------------------------------------------------------ tensor-core fragments
// mma.sync m16n8k16, f16 x f16 -> f32 (row.col).  Used for the 8-head products of the decode
// attention, where N = 8 query heads of one KV head.
__device__ __forceinline__ void mma_f16_16816(float (&c)[4], const uint32_t (&a)[4], const uint32_t (&b)[2]) {
    asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 "
                 "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
                 : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
                 : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]));
}
// Transpose an 8x8 b16 matrix held in the standard fragment layout.
__device__ __forceinline__ uint32_t movmatrix_trans(uint32_t x) {
    uint32_t y;
    asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(y) : "r"(x));
    return y;
}
__device__ __forceinline__ uint32_t pack_f16x2(float lo, float hi) {
    __half2 h = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t *>(&h);
}

// int8 bytes -> exact f16 values: f16x2(byte0, byte2) of a word w of four int8.  Each byte x
// becomes the f16 1024 + (x + 128) (bits 0x6400 | (x ^ 0x80)) and 1152 is subtracted, exactly.
__device__ __forceinline__ uint32_t i8x2_even_to_f16x2(uint32_t w) {
    uint32_t t = (w & 0x00FF00FFu) ^ 0x64806480u;
    __half2 h = __hsub2(*reinterpret_cast<__half2 *>(&t), __halves2half2(__ushort_as_half(0x6480), __ushort_as_half(0x6480)));
    return *reinterpret_cast<uint32_t *>(&h);
}

// The same conversions without the subtraction: each value comes out as the f16 1152 + x
// (exact).  The bias is removed by one more MMA whose A operand is the constant -1152
// (F16X2_NEG1152 in every register): it adds -1152 x (sum of the B column) to every row.
constexpr uint32_t F16X2_NEG1152 = 0xE480E480u;
__device__ __forceinline__ uint32_t i8x2_even_biased(uint32_t w) { return (w & 0x00FF00FFu) ^ 0x64806480u; }
__device__ __forceinline__ uint32_t i8x2_odd_biased(uint32_t w) { return ((w >> 8) & 0x00FF00FFu) ^ 0x64806480u; }
template <int B>
__device__ __forceinline__ uint32_t i8_pair_biased(uint32_t w0, uint32_t w1) {
    return i8x2_even_biased(__byte_perm(w0, w1, B | ((4 + B) << 8)));
}

// 32-bit load from shared memory at a 2-byte aligned address (q8_0 rows are 34-byte strided).
__device__ __forceinline__ uint32_t lds_u32_a2(const uint8_t * p) {
    const uintptr_t a = reinterpret_cast<uintptr_t>(p);
    if ((a & 3u) == 0) return *reinterpret_cast<const uint32_t *>(p);
    const uint32_t * w = reinterpret_cast<const uint32_t *>(a - 2);
    return __funnelshift_r(w[0], w[1], 16);
}

}  // namespace qsa
