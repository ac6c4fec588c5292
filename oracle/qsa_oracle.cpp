// qsa_oracle.cpp -- CPU restatement of QwFNfer's sparse-attention (QSA) node.
//
// TEST INFRASTRUCTURE ONLY.  This file is the parity checker for the CUDA library and the
// timed CPU baseline of bench.py; only tests/, __graft_entry__.smoke() and bench.py's CPU legs
// load it.  The product (libqsa.so) never links, loads or calls it.
//
// The reference computes the node with ggml graph ops (third-party ggml, not in the reference
// tree).  This file restates, op by op, what those graphs compute, citing the reference call
// site for each step.  Where ggml's own arithmetic matters (rounding points, accumulation
// width), the choice made here is stated at the function.  Pinning: q8_0 and f16 rounding are
// checked against gguf-py's codec (which states bit-exactness with ggml-quants.c) by the
// committed fixtures under tests/golden; the bias/selection rules are checked against a literal
// restatement of the reference's host code; the attention against a dense fp64 attention where
// every cell is selected (src/qwfn_graph.h:29-35).
//
// Build: g++ -O3 -march=native -fopenmp -ffp-contract=off -shared -fPIC (see oracle/Makefile).

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <vector>

#include <omp.h>

#include "../include/qsa.h"

namespace {

// ------------------------------------------------------------------ f16 / bf16
// IEEE binary16, round-to-nearest-even (what ggml's GGML_FP32_TO_FP16 does on x86 through F16C,
// and what its software fallback does).
inline uint16_t f32_to_f16(float f) {
    _Float16 h = (_Float16) f;
    uint16_t u;
    std::memcpy(&u, &h, 2);
    return u;
}
inline float f16_to_f32(uint16_t u) {
    _Float16 h;
    std::memcpy(&h, &u, 2);
    return (float) h;
}
inline float bf16_to_f32(uint16_t u) {
    uint32_t w = (uint32_t) u << 16;
    float f;
    std::memcpy(&f, &w, 4);
    return f;
}

// f32 -> bf16 rounded to nearest even (ggml's fp32 -> bf16 conversion; a NaN stays a quiet NaN).
inline uint16_t f32_to_bf16(float f) {
    uint32_t u;
    std::memcpy(&u, &f, 4);
    if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t) ((u >> 16) | 64u);
    return (uint16_t) ((u + (0x7fffu + ((u >> 16) & 1u))) >> 16);
}

constexpr int QK8_0 = 32;
constexpr size_t Q8_0_BYTES = 34;

// ggml quantize_row_q8_0_ref (ggml-quants.c), the rounding gguf-py's Q8_0 reproduces:
// d = amax/127, id = 1/d, q = roundf(x*id) (half away from zero), d stored as f16.
void q8_0_quantize_block(const float * x, uint8_t * out) {
    float amax = 0.0f;
    for (int j = 0; j < QK8_0; j++) amax = std::max(amax, std::fabs(x[j]));
    const float d  = amax / 127.0f;
    const float id = d != 0.0f ? 1.0f / d : 0.0f;
    const uint16_t dh = f32_to_f16(d);
    std::memcpy(out, &dh, 2);
    for (int j = 0; j < QK8_0; j++) {
        const float v = x[j] * id;
        out[2 + j] = (uint8_t) (int8_t) std::roundf(v);
    }
}
inline float q8_0_value(const uint8_t * row, int i) {
    const uint8_t * blk = row + (size_t) (i / QK8_0) * Q8_0_BYTES;
    uint16_t dh;
    std::memcpy(&dh, blk, 2);
    return f16_to_f32(dh) * (float) (int8_t) blk[2 + i % QK8_0];
}

size_t row_bytes(int32_t type, int64_t n) {
    switch (type) {
        case QSA_TYPE_Q8_0: return (size_t) (n / QK8_0) * Q8_0_BYTES;
        case QSA_TYPE_F16:  return (size_t) n * 2;
        case QSA_TYPE_F32:  return (size_t) n * 4;
        default: return 0;
    }
}

// Element i of a K/V cache row (kv_dim elements) as f32.  For q8_0 this is d*q in f32 (ggml's
// dequantize_row_q8_0); `round_f16` then rounds it to f16, as the decode graph's
// ggml_cast(F16) of the gathered rows does (src/qwfn_graph.cpp:531-532).
inline float kv_value(const uint8_t * row, int32_t type, int i, bool round_f16) {
    float v;
    if (type == QSA_TYPE_Q8_0) {
        v = q8_0_value(row, i);
        if (round_f16) v = f16_to_f32(f32_to_f16(v));
    } else {
        uint16_t h;
        std::memcpy(&h, row + (size_t) i * 2, 2);
        v = f16_to_f32(h);
    }
    return v;
}

int64_t n_force_max(const qsa_desc * d) {
    return d->window > 0 ? (d->window + d->ratio - 1) / d->ratio + 1 : 1;
}

}  // namespace

extern "C" {

// Oracle modes for the attention step.
enum {
    ORC_KV_F16_ROUND = 1,  // round dequantized q8_0 K/V to f16 (decode gather, src/qwfn_graph.cpp:531-532)
    ORC_Q_F16        = 2,  // round Q to f16 before the KQ dot (CPU FA converts Q to K's vec_dot type)
    ORC_GGML_FA      = 4,  // ggml CPU flash-attn loop: f32 online softmax in cell order with expf
    ORC_GGML_V_F16   = 8   // ... and with an F16 V accumulator for F16 V (recollection of ggml-cpu)
};

int orc_version(void) { return 1; }
int orc_max_threads(void) { return omp_get_max_threads(); }
void orc_set_threads(int n) { omp_set_num_threads(n > 0 ? n : 1); }

void orc_f32_to_f16(const float * x, uint16_t * y, int64_t n) {
    for (int64_t i = 0; i < n; i++) y[i] = f32_to_f16(x[i]);
}
void orc_f16_to_f32(const uint16_t * x, float * y, int64_t n) {
    for (int64_t i = 0; i < n; i++) y[i] = f16_to_f32(x[i]);
}

// n a multiple of 32.
void orc_q8_0_quantize(const float * x, uint8_t * out, int64_t n) {
    #pragma omp parallel for schedule(static) if (n > (1 << 16))
    for (int64_t b = 0; b < n / QK8_0; b++) q8_0_quantize_block(x + b * QK8_0, out + b * Q8_0_BYTES);
}
void orc_q8_0_dequantize(const uint8_t * q, float * y, int64_t n) {
    #pragma omp parallel for schedule(static) if (n > (1 << 16))
    for (int64_t i = 0; i < n; i++) y[i] = q8_0_value(q + (i / QK8_0) * Q8_0_BYTES, (int) (i % QK8_0));
}

// Append n_tok tokens at pos0: K/V rows quantized to the cache type (ggml_set_rows / ggml_cpy
// F32 -> type_k, src/qwfn_graph.cpp:525-528, 353-360) and the raw indexer key to F16
// (src/qwfn_graph.cpp:469, 251-254).  Any of k/v/kidx may be NULL.
void orc_append(const qsa_desc * d, uint8_t * kc, uint8_t * vc, uint16_t * ic,
                int64_t pos0, int64_t n_tok, const float * k, const float * v, const float * kidx) {
    const int64_t kv_dim = (int64_t) d->n_head_kv * d->head_dim;
    const size_t rbk = row_bytes(d->type_k, kv_dim), rbv = row_bytes(d->type_v, kv_dim);
    #pragma omp parallel for schedule(static) if (n_tok > 64)
    for (int64_t t = 0; t < n_tok; t++) {
        const int64_t row = pos0 + t;
        for (int w = 0; w < 2; w++) {
            const float * src = w == 0 ? k : v;
            if (!src) continue;
            const int32_t ty = w == 0 ? d->type_k : d->type_v;
            uint8_t * dst = (w == 0 ? kc : vc) + (size_t) row * (w == 0 ? rbk : rbv);
            const float * x = src + t * kv_dim;
            if (ty == QSA_TYPE_Q8_0) {
                for (int64_t b = 0; b < kv_dim / QK8_0; b++) q8_0_quantize_block(x + b * QK8_0, dst + b * Q8_0_BYTES);
            } else {
                uint16_t * h = (uint16_t *) dst;
                for (int64_t i = 0; i < kv_dim; i++) h[i] = f32_to_f16(x[i]);
            }
        }
        if (kidx && ic)
            for (int64_t i = 0; i < d->idx_dim; i++) ic[row * d->idx_dim + i] = f32_to_f16(kidx[t * d->idx_dim + i]);
    }
}

// Pooled key of one block, qsa_pool_blocks (src/qwfn_graph.cpp:412-429):
//   sum   = slice_0 + slice_1 + ... + slice_{r-1}     sequential f32 ggml_add (:416-421)
//   mean  = sum * (1/r)                              ggml_scale by the f32 1/r (:422)
//   y     = rms_norm(mean) * k_norm_w                ggml_rms_norm then ggml_mul (:423);
//           rms_norm: sum of x*x (each product f32) accumulated in double, mean = (float)(sum/n),
//           scale = 1/sqrtf(mean+eps) in f32, y = x*scale
//   out   = IMRoPE(y, pos = b*r for every section)   ggml_rope_multi IMROPE (:425-427); the
//           block positions come from src/qwfn_engine.cpp:742 / :776-778 (all sections b*r)
// IMRoPE as ggml's mrope cache: theta_scale = powf(base, -2/rope_dim); per pair i the section
// rule picks t/h/w/e, each position advanced by a chain of f32 multiplies by theta_scale;
// cos/sin of the f32 angle; NEOX pairs (i, i+rope_dim/2); dims >= rope_dim pass through.
void orc_pool_blocks(const qsa_desc * d, const uint16_t * ic, int64_t blk0, int64_t n_blk,
                     const float * k_norm_w, float * out_f32, uint16_t * out_f16) {
    const int64_t D = d->idx_dim, r = d->ratio, nd = d->rope_dim;
    const float theta_scale = powf(d->rope_freq_base, -2.0f / (float) nd);
    const int * s = d->sections;
    const int sect_dims = s[0] + s[1] + s[2] + s[3];
    #pragma omp parallel for schedule(static) if (n_blk > 16)
    for (int64_t j = 0; j < n_blk; j++) {
        const int64_t b = blk0 + j;
        std::vector<float> x(D, 0.0f), y(D);
        for (int64_t i = 0; i < r; i++) {
            const uint16_t * row = ic + (b * r + i) * D;
            for (int64_t e = 0; e < D; e++) x[e] = i == 0 ? f16_to_f32(row[e]) : x[e] + f16_to_f32(row[e]);
        }
        const float inv_r = 1.0f / (float) r;
        for (int64_t e = 0; e < D; e++) x[e] = x[e] * inv_r;
        double ss = 0.0;
        for (int64_t e = 0; e < D; e++) ss += (double) (x[e] * x[e]);
        const float mean  = (float) (ss / (double) D);
        const float scale = 1.0f / sqrtf(mean + d->rms_eps);
        for (int64_t e = 0; e < D; e++) {
            y[e] = x[e] * scale;
            if (k_norm_w) y[e] = y[e] * k_norm_w[e];
        }
        // rope at positions (p, p, p, 0)
        const float p = (float) (b * r);
        float th_t = p, th_h = p, th_w = p, th_e = 0.0f;
        std::vector<float> out(y);
        for (int64_t i0 = 0; i0 < nd; i0 += 2) {
            const int sector = (int) ((i0 / 2) % sect_dims);
            float theta;
            if (sector % 3 == 1 && sector < 3 * s[1])      theta = th_h;
            else if (sector % 3 == 2 && sector < 3 * s[2]) theta = th_w;
            else if (sector % 3 == 0 && sector < 3 * s[0]) theta = th_t;
            else                                           theta = th_e;
            const float c = cosf(theta), sn = sinf(theta);
            const int64_t ic0 = i0 / 2;
            const float x0 = y[ic0], x1 = y[ic0 + nd / 2];
            out[ic0]          = x0 * c - x1 * sn;
            out[ic0 + nd / 2] = x0 * sn + x1 * c;
            th_t *= theta_scale; th_h *= theta_scale; th_w *= theta_scale; th_e *= theta_scale;
        }
        for (int64_t e = 0; e < D; e++) {
            if (out_f32) out_f32[j * D + e] = out[e];
            if (out_f16) out_f16[j * D + e] = f32_to_f16(out[e]);
        }
    }
}

// Indexer scores of n_q queries against blocks [0, nb) of the pooled cache
// (src/qwfn_graph.cpp:485-491, prefill :286-293):
//   per head h: dot = mul_mat(pool F16, q) -- q converted to F16 (the CPU mul_mat converts the
//   f32 operand to the F16 weight's vec_dot type); products of two f16 are exact in f32 and
//   are accumulated here in double and rounded once to f32 (ggml's SIMD f32 lanes agree to a
//   few ulp, which is why selection parity excludes near-ties);
//   relu; sum over heads (ggml_sum_rows: double accumulation, one f32 rounding).
// The bias is not added: selection applies it as a rule (orc_select).
void orc_scores(const qsa_desc * d, const uint16_t * pool, int64_t nb, int64_t n_q,
                const float * q_idx, float * scores /* [n_q][nb] */) {
    const int64_t D = d->idx_dim, H = d->idx_n_head;
    #pragma omp parallel for schedule(static) if (n_q * nb > 4096)
    for (int64_t t = 0; t < n_q; t++) {
        std::vector<float> qh(H * D);
        for (int64_t i = 0; i < H * D; i++) qh[i] = f16_to_f32(f32_to_f16(q_idx[t * H * D + i]));
        for (int64_t b = 0; b < nb; b++) {
            double hs = 0.0;
            for (int64_t h = 0; h < H; h++) {
                double acc = 0.0;
                for (int64_t e = 0; e < D; e++) acc += (double) (f16_to_f32(pool[b * D + e]) * qh[h * D + e]);
                float dot = (float) acc;
                hs += (double) (dot > 0.0f ? dot : 0.0f);
            }
            scores[t * nb + b] = (float) hs;
        }
    }
}

// Selection for the query at position q (src/qwfn_graph.cpp:493-495, prefill :295-306; bias
// rules src/qwfn_engine.cpp:748-753, 936-950; tools/qwfn_logits.cpp:165-176):
//   visible   : blocks whole at q, (b+1)*r <= q+1        (bias 0 in the reference)
//   forced    : window == 0 -> the query's block b_q while it is incomplete at q (bias +1e9);
//               window  > 0 -> blocks b_q-nf+1 .. b_q, nf = ceil(window/r)+1 (bias +1e9)
//   others    : blocks after q (-1e9) or past the cache (-inf): never useful (masked cells)
//   kept      : forced, then the KB-|forced| highest-scoring visible non-forced blocks,
//               KB = top_k_blocks + nf (nf = 1 when window == 0); equal scores -> lower index.
// This is ggml_top_k(score + bias, KB) for every input where the k-th and (k+1)-th visible
// scores differ.  Output: block ids ascending, -1 padded to KB; returns the count.
int orc_select(const qsa_desc * d, const float * scores, int64_t q, int32_t * sel, uint8_t * is_forced) {
    const int64_t r = d->ratio, KB = d->top_k_blocks + n_force_max(d);
    const int64_t bq = q / r, n_vis = (q + 1) / r;
    std::vector<int64_t> forced;
    if (d->window > 0) {
        for (int64_t b = std::max<int64_t>(0, bq - n_force_max(d) + 1); b <= bq; b++) forced.push_back(b);
    } else if ((q + 1) % r != 0) {
        forced.push_back(bq);
    }
    std::vector<int64_t> cand;
    for (int64_t b = 0; b < n_vis; b++)
        if (std::find(forced.begin(), forced.end(), b) == forced.end()) cand.push_back(b);
    const int64_t want = std::max<int64_t>(0, KB - (int64_t) forced.size());
    std::stable_sort(cand.begin(), cand.end(), [&](int64_t a, int64_t b) { return scores[a] > scores[b]; });
    if ((int64_t) cand.size() > want) cand.resize(want);
    std::vector<int64_t> all(forced);
    all.insert(all.end(), cand.begin(), cand.end());
    std::sort(all.begin(), all.end());
    int n = 0;
    for (int64_t i = 0; i < KB; i++) {
        sel[i] = i < (int64_t) all.size() ? (int32_t) all[i] : -1;
        if (is_forced) is_forced[i] = i < (int64_t) all.size() &&
            std::find(forced.begin(), forced.end(), all[i]) != forced.end();
        if (i < (int64_t) all.size()) n++;
    }
    return n;
}

// Attention of n_q queries, each over the cells c <= q_pos of its selected blocks
// (ggml_flash_attn_ext, scale 1/sqrt(head_dim), GQA head h -> KV head h/(n_head/n_head_kv),
// src/qwfn_graph.cpp:539-541, prefill :400-403).
//   default      : K.Q in double, softmax and V accumulation in double (exact reference)
//   ORC_GGML_FA  : ggml-cpu's loop -- for each cell in order: s = dot*scale; online max M,
//                  sum S (f32, expf); V accumulated in f32, or in f16 with ORC_GGML_V_F16
// Q is f32 or bf16 [n_q][n_head][head_dim]; out f32 [n_q][n_head][head_dim].
void orc_attend(const qsa_desc * d, const uint8_t * kc, const uint8_t * vc,
                int64_t n_q, const int64_t * q_pos, const int32_t * sel, int64_t sel_stride,
                const void * Q, int32_t q_type, float * out, int32_t flags) {
    const int64_t hd = d->head_dim, nh = d->n_head, nkv = d->n_head_kv, gqa = nh / nkv, r = d->ratio;
    const int64_t kv_dim = nkv * hd;
    const size_t rbk = row_bytes(d->type_k, kv_dim), rbv = row_bytes(d->type_v, kv_dim);
    const bool kv_round = flags & ORC_KV_F16_ROUND, q_f16 = flags & ORC_Q_F16;
    const float scale = 1.0f / sqrtf((float) hd);
    #pragma omp parallel for schedule(dynamic) collapse(2)
    for (int64_t t = 0; t < n_q; t++) {
        for (int64_t h = 0; h < nh; h++) {
            const int64_t g = h / gqa, qp = q_pos[t];
            std::vector<float> qv(hd);
            for (int64_t e = 0; e < hd; e++) {
                const int64_t idx = (t * nh + h) * hd + e;
                float x = q_type == QSA_TYPE_BF16 ? bf16_to_f32(((const uint16_t *) Q)[idx]) : ((const float *) Q)[idx];
                qv[e] = q_f16 ? f16_to_f32(f32_to_f16(x)) : x;
            }
            std::vector<int64_t> cells;
            for (int64_t i = 0; i < sel_stride; i++) {
                const int32_t b = sel[t * sel_stride + i];
                if (b < 0) continue;
                for (int64_t c = b * r; c < (b + 1) * r && c <= qp; c++) cells.push_back(c);
            }
            float * o = out + (t * nh + h) * hd;
            std::vector<float> kf(hd), vf(hd);
            if (!(flags & ORC_GGML_FA)) {
                std::vector<double> s(cells.size());
                double m = -INFINITY;
                for (size_t j = 0; j < cells.size(); j++) {
                    const uint8_t * kr = kc + (size_t) cells[j] * rbk;
                    double acc = 0.0;
                    for (int64_t e = 0; e < hd; e++) acc += (double) kv_value(kr, d->type_k, (int) (g * hd + e), kv_round) * (double) qv[e];
                    s[j] = acc * (double) scale;
                    m = std::max(m, s[j]);
                }
                std::vector<double> acc(hd, 0.0);
                double l = 0.0;
                for (size_t j = 0; j < cells.size(); j++) {
                    const double p = std::exp(s[j] - m);
                    l += p;
                    const uint8_t * vr = vc + (size_t) cells[j] * rbv;
                    for (int64_t e = 0; e < hd; e++) acc[e] += p * (double) kv_value(vr, d->type_v, (int) (g * hd + e), kv_round);
                }
                for (int64_t e = 0; e < hd; e++) o[e] = l > 0.0 ? (float) (acc[e] / l) : 0.0f;
            } else {
                const bool v16 = (flags & ORC_GGML_V_F16) != 0;
                std::vector<float> acc32(hd, 0.0f);
                std::vector<uint16_t> acc16(hd, 0);
                float M = -INFINITY, S = 0.0f;
                for (size_t j = 0; j < cells.size(); j++) {
                    const uint8_t * kr = kc + (size_t) cells[j] * rbk;
                    double a = 0.0;
                    for (int64_t e = 0; e < hd; e++) a += (double) (kv_value(kr, d->type_k, (int) (g * hd + e), kv_round) * qv[e]);
                    const float sc = (float) a * scale;
                    const float Mold = M;
                    float ms = 1.0f, vs = 1.0f;
                    const uint8_t * vr = vc + (size_t) cells[j] * rbv;
                    if (sc > M) {
                        M = sc;
                        ms = expf(Mold - M);
                        if (v16) for (int64_t e = 0; e < hd; e++) acc16[e] = f32_to_f16(f16_to_f32(acc16[e]) * ms);
                        else     for (int64_t e = 0; e < hd; e++) acc32[e] *= ms;
                    } else {
                        vs = expf(sc - M);
                    }
                    for (int64_t e = 0; e < hd; e++) {
                        const float vv = kv_value(vr, d->type_v, (int) (g * hd + e), kv_round);
                        if (v16) acc16[e] = f32_to_f16(fmaf(vv, vs, f16_to_f32(acc16[e])));
                        else     acc32[e] = fmaf(vv, vs, acc32[e]);
                    }
                    S = S * ms + vs;
                }
                const float Sinv = S == 0.0f ? 0.0f : 1.0f / S;
                for (int64_t e = 0; e < hd; e++) o[e] = (v16 ? f16_to_f32(acc16[e]) : acc32[e]) * Sinv;
            }
        }
    }
}

// Unnormalised attention state of n_q queries over their selected blocks, the layout the
// sharded decode exchanges between devices: per query 16 rows (KV head g, query head h of its
// group -> row 8g+h; unused rows M=-inf, L=0, O=0), as [M 16][L 16][O 16 x head_dim] with
//   M = max_c s_c * log2(e) / sqrt(head_dim)   (log2 domain),
//   L = sum_c 2^(s'_c - M),  O = sum_c 2^(s'_c - M) v_c.
// Computed in double (exact reference arithmetic) and rounded once; an empty selection gives
// M = -inf.  Merging states of disjoint cell sets reproduces orc_attend's output.
void orc_attend_state(const qsa_desc * d, const uint8_t * kc, const uint8_t * vc,
                      int64_t n_q, const int64_t * q_pos, const int32_t * sel, int64_t sel_stride,
                      const void * Q, int32_t q_type, float * state, int32_t flags) {
    const int64_t hd = d->head_dim, nh = d->n_head, nkv = d->n_head_kv, gqa = nh / nkv, r = d->ratio;
    const int64_t kv_dim = nkv * hd, SF = 2 * 16 + 16 * hd;
    const size_t rbk = row_bytes(d->type_k, kv_dim), rbv = row_bytes(d->type_v, kv_dim);
    const bool kv_round = flags & ORC_KV_F16_ROUND, q_f16 = flags & ORC_Q_F16;
    const double scale_log2 = 1.4426950408889634 / std::sqrt((double) hd);
    #pragma omp parallel for schedule(dynamic) collapse(2)
    for (int64_t t = 0; t < n_q; t++) {
        for (int64_t row = 0; row < 16; row++) {
            float * st = state + t * SF;
            const int64_t g = row / 8, h = row % 8;
            float * o = st + 32 + row * hd;
            if (g >= nkv || h >= gqa) {
                st[row] = -INFINITY; st[16 + row] = 0.0f;
                for (int64_t e = 0; e < hd; e++) o[e] = 0.0f;
                continue;
            }
            const int64_t head = g * gqa + h, qp = q_pos[t];
            std::vector<float> qv(hd);
            for (int64_t e = 0; e < hd; e++) {
                const int64_t idx = (t * nh + head) * hd + e;
                float x = q_type == QSA_TYPE_BF16 ? bf16_to_f32(((const uint16_t *) Q)[idx]) : ((const float *) Q)[idx];
                qv[e] = q_f16 ? f16_to_f32(f32_to_f16(x)) : x;
            }
            std::vector<int64_t> cells;
            for (int64_t i = 0; i < sel_stride; i++) {
                const int32_t b = sel[t * sel_stride + i];
                if (b < 0) continue;
                for (int64_t c = b * r; c < (b + 1) * r && c <= qp; c++) cells.push_back(c);
            }
            std::vector<double> s(cells.size());
            double m = -INFINITY;
            for (size_t j = 0; j < cells.size(); j++) {
                const uint8_t * kr = kc + (size_t) cells[j] * rbk;
                double acc = 0.0;
                for (int64_t e = 0; e < hd; e++) acc += (double) kv_value(kr, d->type_k, (int) (g * hd + e), kv_round) * (double) qv[e];
                s[j] = acc * scale_log2;
                m = std::max(m, s[j]);
            }
            std::vector<double> acc(hd, 0.0);
            double l = 0.0;
            for (size_t j = 0; j < cells.size(); j++) {
                const double p = std::exp2(s[j] - m);
                l += p;
                const uint8_t * vr = vc + (size_t) cells[j] * rbv;
                for (int64_t e = 0; e < hd; e++) acc[e] += p * (double) kv_value(vr, d->type_v, (int) (g * hd + e), kv_round);
            }
            st[row] = (float) m;
            st[16 + row] = (float) l;
            for (int64_t e = 0; e < hd; e++) o[e] = (float) acc[e];
        }
    }
}

// Blocks kept per query (KB).
int orc_k_blocks(const qsa_desc * d) { return (int) (d->top_k_blocks + n_force_max(d)); }

// The whole node for n_q queries over one cache whose pooled keys are current: scores over the
// blocks whole at each query, selection, attention.  sel (int32 [n_q][KB]) receives the
// selection; scores_out (optional, [n_q][nb]) the raw head-summed scores.
void orc_node(const qsa_desc * d, const uint8_t * kc, const uint8_t * vc, const uint16_t * pool,
              int64_t n_q, const int64_t * q_pos, const void * Q, int32_t q_type, const float * q_idx,
              float * out, int32_t * sel, float * scores_out, int32_t flags) {
    const int64_t KB = orc_k_blocks(d);
    int64_t nb_max = 0;
    for (int64_t t = 0; t < n_q; t++) nb_max = std::max<int64_t>(nb_max, (q_pos[t] + 1) / d->ratio);
    const int64_t nb = std::max<int64_t>(nb_max, 1);
    std::vector<float> sc((size_t) n_q * nb, 0.0f);
    if (nb_max > 0) orc_scores(d, pool, nb_max, n_q, q_idx, sc.data());
    for (int64_t t = 0; t < n_q; t++) {
        orc_select(d, sc.data() + t * nb, q_pos[t], sel + t * KB, nullptr);
        if (scores_out) std::memcpy(scores_out + t * nb, sc.data() + t * nb, (size_t) nb * 4);
    }
    orc_attend(d, kc, vc, n_q, q_pos, sel, KB, Q, q_type, out, flags);
}


// rms_norm * w then IMRoPE at position `pos` over one head of D values, in place: the arithmetic
// of orc_pool_blocks's norm and rope (rms(): ggml_rms_norm then ggml_mul, src/qwfn_graph.cpp:114-115;
// ggml_rope_multi IMROPE with positions (p, p, p, 0)).
static void orc_norm_rope(const qsa_desc * d, float * v, int64_t D, const float * w, float pos) {
    const int64_t nd = d->rope_dim;
    const float theta_scale = powf(d->rope_freq_base, -2.0f / (float) nd);
    const int * s = d->sections;
    const int sect_dims = s[0] + s[1] + s[2] + s[3];
    double ss = 0.0;
    for (int64_t e = 0; e < D; e++) ss += (double) (v[e] * v[e]);
    const float mean  = (float) (ss / (double) D);
    const float scale = 1.0f / sqrtf(mean + d->rms_eps);
    std::vector<float> y(D);
    for (int64_t e = 0; e < D; e++) {
        y[e] = v[e] * scale;
        if (w) y[e] = y[e] * w[e];
    }
    float th_t = pos, th_h = pos, th_w = pos, th_e = 0.0f;
    for (int64_t e = 0; e < D; e++) v[e] = y[e];
    for (int64_t i0 = 0; i0 < nd; i0 += 2) {
        const int sector = (int) ((i0 / 2) % sect_dims);
        float theta;
        if (sector % 3 == 1 && sector < 3 * s[1])      theta = th_h;
        else if (sector % 3 == 2 && sector < 3 * s[2]) theta = th_w;
        else if (sector % 3 == 0 && sector < 3 * s[0]) theta = th_t;
        else                                           theta = th_e;
        const float c = cosf(theta), sn = sinf(theta);
        const int64_t ic0 = i0 / 2;
        const float x0 = y[ic0], x1 = y[ic0 + nd / 2];
        v[ic0]          = x0 * c - x1 * sn;
        v[ic0 + nd / 2] = x0 * sn + x1 * c;
        th_t *= theta_scale; th_h *= theta_scale; th_w *= theta_scale; th_e *= theta_scale;
    }
}

// The projections feeding the node for T tokens (src/qwfn_graph.cpp:465, 479-484, 505-518):
//   y = mul_mat(W bf16, x): x rounded to bf16 (the CPU mul_mat converts the f32 operand to the
//   weight's dot type), products of two bf16 exact in f32, accumulated in double and rounded
//   once to f32 (ggml's f32 SIMD lanes agree to a few ulp);
//   attn_q rows per head h: [2h*hd, 2h*hd+hd) the query, the next hd the gate (:505-510);
//   Q = rms(Q_h)*q_norm, K = rms(K_h)*k_norm, q_idx = rms(q_h)*q_idx_norm, each then IMRoPE at the
//   token's position; V, the gate and the raw indexer key as projected.
// One projection row: bf16 weights (ggml's vec_dot_bf16: the activation rounded to bf16, exact
// f32 products, here summed in double and rounded once), or q8_0 weights (ggml_vec_dot_q8_0_q8_0:
// the activation row quantised to q8_0 with the reference rounding, per block the integer sum of
// products times f32(d_w) * f32(d_x), the block terms summed in double and rounded once).
struct ProjRow {
    int32_t w_type;
    int64_t n;                       // row length (n_embd or n_head*head_dim)
    std::vector<float> xb;           // bf16 path: the activation's bf16 values
    std::vector<uint8_t> xq;         // q8_0 path: the activation's q8_0 blocks
    void set_x(const float * x) {
        if (w_type == QSA_TYPE_Q8_0) {
            xq.resize((size_t) n / QK8_0 * Q8_0_BYTES);
            for (int64_t b = 0; b < n / QK8_0; b++) q8_0_quantize_block(x + b * QK8_0, xq.data() + b * Q8_0_BYTES);
        } else {
            xb.resize((size_t) n);
            for (int64_t e = 0; e < n; e++) xb[e] = bf16_to_f32(f32_to_bf16(x[e]));
        }
    }
    size_t row_bytes() const { return w_type == QSA_TYPE_Q8_0 ? (size_t) n / QK8_0 * Q8_0_BYTES : (size_t) n * 2; }
    float dot(const void * w_base, int64_t row) const {
        const uint8_t * w = static_cast<const uint8_t *>(w_base) + (size_t) row * row_bytes();
        double acc = 0.0;
        if (w_type == QSA_TYPE_Q8_0) {
            for (int64_t b = 0; b < n / QK8_0; b++) {
                const uint8_t * wb = w + b * Q8_0_BYTES, * xb8 = xq.data() + b * Q8_0_BYTES;
                uint16_t dw, dx;
                std::memcpy(&dw, wb, 2);
                std::memcpy(&dx, xb8, 2);
                int32_t sumi = 0;
                for (int j = 0; j < QK8_0; j++) sumi += (int32_t) (int8_t) wb[2 + j] * (int32_t) (int8_t) xb8[2 + j];
                acc += (double) ((float) sumi * (f16_to_f32(dw) * f16_to_f32(dx)));
            }
        } else {
            const uint16_t * wr = reinterpret_cast<const uint16_t *>(w);
            for (int64_t e = 0; e < n; e++) acc += (double) (bf16_to_f32(wr[e]) * xb[e]);
        }
        return (float) acc;
    }
};

void orc_front_w(const qsa_desc * d, int32_t w_type, const void * wq, const void * wk, const void * wv,
                 const void * wq_idx, const void * wk_idx, const float * q_norm, const float * k_norm,
                 const float * q_idx_norm, int64_t n_embd, int64_t T, const int32_t * pos, const float * x,
                 float * q_out, float * gate_out, float * q_idx_out, float * k_out, float * v_out, float * kidx_out) {
    const int64_t hd = d->head_dim, nh = d->n_head, nkv = d->n_head_kv, H = d->idx_n_head, D = d->idx_dim;
    #pragma omp parallel for schedule(static) if (T > 1)
    for (int64_t t = 0; t < T; t++) {
        ProjRow pr{w_type, n_embd, {}, {}};
        pr.set_x(x + t * n_embd);
        std::vector<float> v(hd);
        const float p = (float) pos[t];
        for (int64_t h = 0; h < nh; h++) {
            for (int64_t e = 0; e < hd; e++) v[e] = pr.dot(wq, 2 * h * hd + e);
            orc_norm_rope(d, v.data(), hd, q_norm, p);
            std::memcpy(q_out + (t * nh + h) * hd, v.data(), (size_t) hd * 4);
            for (int64_t e = 0; e < hd; e++) gate_out[(t * nh + h) * hd + e] = pr.dot(wq, (2 * h + 1) * hd + e);
        }
        for (int64_t j = 0; j < nkv; j++) {
            for (int64_t e = 0; e < hd; e++) v[e] = pr.dot(wk, j * hd + e);
            orc_norm_rope(d, v.data(), hd, k_norm, p);
            std::memcpy(k_out + (t * nkv + j) * hd, v.data(), (size_t) hd * 4);
            for (int64_t e = 0; e < hd; e++) v_out[(t * nkv + j) * hd + e] = pr.dot(wv, j * hd + e);
        }
        std::vector<float> qi(D);
        for (int64_t h = 0; h < H; h++) {
            for (int64_t e = 0; e < D; e++) qi[e] = pr.dot(wq_idx, h * D + e);
            orc_norm_rope(d, qi.data(), D, q_idx_norm, p);
            std::memcpy(q_idx_out + (t * H + h) * D, qi.data(), (size_t) D * 4);
        }
        for (int64_t e = 0; e < D; e++) kidx_out[t * D + e] = pr.dot(wk_idx, e);
    }
}

void orc_front(const qsa_desc * d, const uint16_t * wq, const uint16_t * wk, const uint16_t * wv,
               const uint16_t * wq_idx, const uint16_t * wk_idx, const float * q_norm, const float * k_norm,
               const float * q_idx_norm, int64_t n_embd, int64_t T, const int32_t * pos, const float * x,
               float * q_out, float * gate_out, float * q_idx_out, float * k_out, float * v_out, float * kidx_out) {
    orc_front_w(d, QSA_TYPE_BF16, wq, wk, wv, wq_idx, wk_idx, q_norm, k_norm, q_idx_norm, n_embd, T, pos, x,
                q_out, gate_out, q_idx_out, k_out, v_out, kidx_out);
}


// The output side (src/qwfn_graph.cpp:543-545): z = attn * sigmoid(gate) in f32 (ggml_sigmoid:
// 1/(1+expf(-g))), then mul_mat(attn_output, z) as ProjRow computes it (bf16 or q8_0 weights).
void orc_output_w(const qsa_desc * d, int32_t w_type, const void * wo, int64_t n_embd, int64_t T, const float * attn,
                  const float * gate, float * y) {
    const int64_t n_in = (int64_t) d->n_head * d->head_dim;
    #pragma omp parallel for schedule(static) if (T > 1)
    for (int64_t t = 0; t < T; t++) {
        std::vector<float> z(n_in);
        for (int64_t e = 0; e < n_in; e++) {
            const float sg = 1.0f / (1.0f + expf(-gate[t * n_in + e]));
            z[e] = attn[t * n_in + e] * sg;
        }
        ProjRow pr{w_type, n_in, {}, {}};
        pr.set_x(z.data());
        for (int64_t r = 0; r < n_embd; r++) y[t * n_embd + r] = pr.dot(wo, r);
    }
}

void orc_output(const qsa_desc * d, const uint16_t * wo, int64_t n_embd, int64_t T, const float * attn,
                const float * gate, float * y) {
    orc_output_w(d, QSA_TYPE_BF16, wo, n_embd, T, attn, gate, y);
}

}  // extern "C"
