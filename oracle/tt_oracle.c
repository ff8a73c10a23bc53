/*
 * tt_oracle.c -- TEST INFRASTRUCTURE ONLY (see tt_oracle.h).
 *
 * Plain-C restatement of the reference TriTierCache algorithms.  Paths below
 * are relative to the reference project root.  Vector-lane semantics of the
 * reference's AVX2 code are restated explicitly where they change results:
 *   - MINPS/MAXPS return the second operand on ties and NaNs:
 *       min(a,b) = a < b ? a : b,  max(a,b) = a > b ? a : b;
 *     std::min/std::max return the first operand on ties:
 *       std::min(a,b) = b < a ? b : a,  std::max(a,b) = a < b ? b : a.
 *   - CVTPS2DQ rounds to nearest even and yields INT_MIN when out of range.
 *   - GCC compiles C++ with -ffp-contract=fast by default (also under
 *     -std=c++17) and the reference is built with -mfma, so the scalar
 *     `a * b + c` forms of the dequant tail, the axpy tail and the decayed
 *     score update are single fused multiply-adds (fmaf() here).  The
 *     dot-product tail `sum += a[i] * b[i]` is not fused by the compiler
 *     (checked against the reference build with head_dim 12/20/36).
 * Build with -O2 -ffp-contract=off (oracle/Makefile) so that nothing else
 * is fused.
 */
#include "tt_oracle.h"
#include <math.h>
#include <stdlib.h>
#include <string.h>
#include <limits.h>
#include <float.h>

/* ------------------------------------------------------------------ */
/* binary16                                                            */
/* ------------------------------------------------------------------ */
uint16_t orc_f32_to_f16(float f) {
    uint32_t x;
    memcpy(&x, &f, 4);
    uint32_t sign = (x >> 16) & 0x8000u;
    uint32_t exp = (x >> 23) & 0xFFu;
    uint32_t man = x & 0x7FFFFFu;
    if (exp == 0xFFu) {
        if (man) return (uint16_t)(sign | 0x7E00u | (man >> 13)); /* quiet NaN */
        return (uint16_t)(sign | 0x7C00u);
    }
    if (exp == 0) return (uint16_t)sign; /* |f| < 2^-126 rounds to zero */
    int e = (int)exp - 127 + 15;
    if (e >= 31) return (uint16_t)(sign | 0x7C00u);
    if (e >= 1) {
        uint32_t base = ((uint32_t)e << 10) | (man >> 13);
        uint32_t rem = man & 0x1FFFu;
        if (rem > 0x1000u || (rem == 0x1000u && (base & 1u))) base += 1u; /* may carry to inf */
        return (uint16_t)(sign | base);
    }
    /* subnormal half: value = m * 2^(exp-150), unit 2^-24 */
    uint32_t m = man | 0x800000u;
    int shift = 14 - e;
    if (shift > 24) return (uint16_t)sign;
    uint32_t q = m >> shift;
    uint32_t rem = m & ((1u << shift) - 1u);
    uint32_t half = 1u << (shift - 1);
    if (rem > half || (rem == half && (q & 1u))) q += 1u;
    return (uint16_t)(sign | q);
}

float orc_f16_to_f32(uint16_t h) {
    uint32_t sign = ((uint32_t)h & 0x8000u) << 16;
    uint32_t exp = ((uint32_t)h >> 10) & 0x1Fu;
    uint32_t man = (uint32_t)h & 0x3FFu;
    uint32_t x;
    if (exp == 0) {
        if (man == 0) {
            x = sign;
        } else { /* subnormal: normalise */
            int e = -1;
            do { man <<= 1; e++; } while (!(man & 0x400u));
            man &= 0x3FFu;
            x = sign | ((uint32_t)(127 - 15 - e) << 23) | (man << 13);
        }
    } else if (exp == 0x1Fu) {
        x = sign | 0x7F800000u | (man << 13);
    } else {
        x = sign | ((exp - 15 + 127) << 23) | (man << 13);
    }
    float f;
    memcpy(&f, &x, 4);
    return f;
}

static inline float vmin_ps(float a, float b) { return a < b ? a : b; }  /* MINPS */
static inline float vmax_ps(float a, float b) { return a > b ? a : b; }  /* MAXPS */
static inline float std_min(float a, float b) { return b < a ? b : a; }  /* std::min */
static inline float std_max(float a, float b) { return a < b ? b : a; }  /* std::max */

/* CVTPS2DQ under the default MXCSR (round to nearest even). */
static inline int32_t cvtps_epi32(float x) {
    if (!(x >= -2147483648.0f && x < 2147483648.0f)) return INT_MIN;
    return (int32_t)nearbyintf(x);
}

static inline void store_meta(void* base, size_t idx, float v, int fp16) {
    if (fp16) ((uint16_t*)base)[idx] = orc_f32_to_f16(v);
    else ((float*)base)[idx] = v;
}
static inline float load_meta(const void* base, size_t idx, int fp16) {
    if (fp16) return orc_f16_to_f32(((const uint16_t*)base)[idx]);
    return ((const float*)base)[idx];
}

/* ------------------------------------------------------------------ */
/* K quantize: csrc/cpu/quantize_k_avx2.cpp:26-110                      */
/* per (head, channel): min/max over the k_group tokens, scale =        */
/* max((max-min)/3, 1e-9), code = clamp(rne((x-min)/scale), 0, 3),      */
/* 16 tokens per word at bit 2*sub_t, word index (w*H + h)*D + c.       */
/* ------------------------------------------------------------------ */
void orc_quantize_k_block(const float* K, uint32_t* packed, void* scale_out, void* zero_out,
                          int meta_fp16, int num_heads, int head_dim, int k_group_size) {
    const int row_stride = num_heads * head_dim;
    const int c_vec_end = (head_dim / 8) * 8;
    const int num_words = k_group_size / 16;
    for (int h = 0; h < num_heads; ++h) {
        const float* hk = K + (size_t)h * head_dim;
        for (int c = 0; c < head_dim; ++c) {
            const int vec = c < c_vec_end;
            float mn = INFINITY, mx = -INFINITY, scale;
            for (int t = 0; t < k_group_size; ++t) {
                float x = hk[(size_t)t * row_stride + c];
                if (vec) { mn = vmin_ps(mn, x); mx = vmax_ps(mx, x); }  /* :48-52 */
                else { mn = std_min(mn, x); mx = std_max(mx, x); }       /* :86-90 */
            }
            if (vec) scale = vmax_ps((mx - mn) / 3.0f, 1e-9f);          /* :54-56 */
            else scale = std_max((mx - mn) / 3.0f, 1e-9f);              /* :92 */
            store_meta(scale_out, (size_t)h * head_dim + c, scale, meta_fp16);
            store_meta(zero_out, (size_t)h * head_dim + c, mn, meta_fp16);
            for (int w = 0; w < num_words; ++w) {
                uint32_t bits = 0;
                for (int sub_t = 0; sub_t < 16; ++sub_t) {
                    float x = hk[(size_t)(w * 16 + sub_t) * row_stride + c];
                    int32_t q = cvtps_epi32((x - mn) / scale);
                    if (q < 0) q = 0;
                    if (q > 3) q = 3;
                    bits |= (uint32_t)q << (2 * sub_t);
                }
                packed[((size_t)w * num_heads + h) * head_dim + c] = bits;
            }
        }
    }
}

/* ------------------------------------------------------------------ */
/* V quantize: csrc/cpu/quantize_v_avx2.cpp:44-108                      */
/* per (token, head): min/max over channels (8-lane tree, hmin8/hmax8   */
/* :7-23), scale as for K, 16 channels per word at bit 2*i, word index  */
/* (t*H + h)*Dq + g.  Requires head_dim % 16 == 0: the reference reads  */
/* v[16g+8 .. 16g+15] unconditionally (:91-92).                          */
/* ------------------------------------------------------------------ */
static float hmin8(const float* v) {
    float m[4], r;
    for (int i = 0; i < 4; ++i) m[i] = vmin_ps(v[i], v[i + 4]);
    float a0 = vmin_ps(m[0], m[2]), a1 = vmin_ps(m[1], m[3]);
    r = vmin_ps(a0, a1);
    return r;
}
static float hmax8(const float* v) {
    float m[4], r;
    for (int i = 0; i < 4; ++i) m[i] = vmax_ps(v[i], v[i + 4]);
    float a0 = vmax_ps(m[0], m[2]), a1 = vmax_ps(m[1], m[3]);
    r = vmax_ps(a0, a1);
    return r;
}

void orc_quantize_v_block(const float* V, int32_t* packed, void* scale_out, void* zero_out,
                          int meta_fp16, int num_heads, int head_dim, int chunk_size) {
    const int qhd = (head_dim + 15) / 16;
    const int row_stride = num_heads * head_dim;
    for (int t = 0; t < chunk_size; ++t) {
        for (int h = 0; h < num_heads; ++h) {
            const float* v = V + (size_t)t * row_stride + (size_t)h * head_dim;
            float mn = INFINITY, mx = -INFINITY;
            int c = 0;
            for (; c + 8 <= head_dim; c += 8) {
                mn = std_min(mn, hmin8(v + c));
                mx = std_max(mx, hmax8(v + c));
            }
            for (; c < head_dim; ++c) {
                mn = std_min(mn, v[c]);
                mx = std_max(mx, v[c]);
            }
            float scale = std_max((mx - mn) / 3.0f, 1e-9f);
            store_meta(scale_out, (size_t)t * num_heads + h, scale, meta_fp16);
            store_meta(zero_out, (size_t)t * num_heads + h, mn, meta_fp16);
            for (int g = 0; g < qhd; ++g) {
                uint32_t word = 0;
                for (int i = 0; i < 16; ++i) {
                    int32_t q = cvtps_epi32((v[g * 16 + i] - mn) / scale);
                    if (q > 3) q = 3;
                    if (q < 0) q = 0;
                    word |= (uint32_t)q << (2 * i);
                }
                packed[((size_t)t * num_heads + h) * qhd + g] = (int32_t)word;
            }
        }
    }
}

/* ------------------------------------------------------------------ */
/* dequantize: csrc/cpu/dequantize_avx2.cpp:24-110 (K), :138-204 (V)    */
/* ------------------------------------------------------------------ */
void orc_dequantize_k(const int32_t* packed, const void* scale, const void* zero, float* out,
                      int meta_fp16, int num_blocks, int num_heads, int head_dim, int k_group_size) {
    const int words = k_group_size / 16;
    const size_t bps = (size_t)words * num_heads * head_dim;
    const size_t bms = (size_t)num_heads * head_dim;
    const size_t ors = (size_t)num_heads * head_dim;
    const int c_vec_end = (head_dim / 8) * 8;
    for (int b = 0; b < num_blocks; ++b)
        for (int h = 0; h < num_heads; ++h)
            for (int c = 0; c < head_dim; ++c) {
                float s = load_meta(scale, b * bms + (size_t)h * head_dim + c, meta_fp16);
                float z = load_meta(zero, b * bms + (size_t)h * head_dim + c, meta_fp16);
                for (int w = 0; w < words; ++w) {
                    int32_t p = packed[b * bps + ((size_t)w * num_heads + h) * head_dim + c];
                    for (int st = 0; st < 16; ++st) {
                        int q = (int)(((uint32_t)p >> (2 * st)) & 3u);
                        size_t tok = (size_t)b * k_group_size + w * 16 + st;
                        float x = fmaf((float)q, s, z);   /* :65, :85, :104 */
                        out[tok * ors + (size_t)h * head_dim + c] = x;
                    }
                }
            }
}

void orc_dequantize_v(const int32_t* packed, const void* scale, const void* zero, float* out,
                      int meta_fp16, int total_tokens, int num_heads, int head_dim) {
    const int qhd = (head_dim + 15) / 16;
    for (int t = 0; t < total_tokens; ++t)
        for (int h = 0; h < num_heads; ++h) {
            float s = load_meta(scale, (size_t)t * num_heads + h, meta_fp16);
            float z = load_meta(zero, (size_t)t * num_heads + h, meta_fp16);
            const int32_t* hp = packed + ((size_t)t * num_heads + h) * qhd;
            float* o = out + ((size_t)t * num_heads + h) * head_dim;
            for (int g = 0; g < qhd; ++g)
                for (int i = 0; i < 16 && g * 16 + i < head_dim; ++i) {
                    int q = (int)(((uint32_t)hp[g] >> (2 * i)) & 3u);
                    o[g * 16 + i] = fmaf((float)q, s, z);
                }
        }
}

/* ------------------------------------------------------------------ */
/* dot_avx2 / axpy_avx2: csrc/cpu/fused_attn_avx2.cpp:11-136            */
/* Eight 8-lane FMA accumulators, pairwise combine, hsum8 tree, then a  */
/* scalar tail (mul, add).                                             */
/* ------------------------------------------------------------------ */
static float dot8(const float* a, const float* b, int n) {
    float acc[8][8];
    memset(acc, 0, sizeof(acc));
    int i = 0;
    for (; i + 64 <= n; i += 64)
        for (int j = 0; j < 8; ++j)
            for (int l = 0; l < 8; ++l) acc[j][l] = fmaf(a[i + 8 * j + l], b[i + 8 * j + l], acc[j][l]);
    for (; i + 32 <= n; i += 32)
        for (int j = 0; j < 4; ++j)
            for (int l = 0; l < 8; ++l) acc[j][l] = fmaf(a[i + 8 * j + l], b[i + 8 * j + l], acc[j][l]);
    for (; i + 8 <= n; i += 8)
        for (int l = 0; l < 8; ++l) acc[0][l] = fmaf(a[i + l], b[i + l], acc[0][l]);
    for (int l = 0; l < 8; ++l) {
        acc[0][l] = acc[0][l] + acc[1][l];
        acc[2][l] = acc[2][l] + acc[3][l];
        acc[4][l] = acc[4][l] + acc[5][l];
        acc[6][l] = acc[6][l] + acc[7][l];
        acc[0][l] = acc[0][l] + acc[2][l];
        acc[4][l] = acc[4][l] + acc[6][l];
        acc[0][l] = acc[0][l] + acc[4][l];
    }
    float s[4];
    for (int l = 0; l < 4; ++l) s[l] = acc[0][l] + acc[0][l + 4];
    float s0 = s[0] + s[2], s1 = s[1] + s[3];
    float sum = s0 + s1;
    for (; i < n; ++i) { float pr = a[i] * b[i]; sum = sum + pr; }   /* :59 */
    return sum;
}

static void axpy8(float* out, const float* x, float scale, int n) {
    int vec_end = (n / 8) * 8;
    for (int i = 0; i < vec_end; ++i) out[i] = fmaf(x[i], scale, out[i]);
    for (int i = vec_end; i < n; ++i) out[i] = fmaf(scale, x[i], out[i]);   /* :135 */
}

/* ------------------------------------------------------------------ */
/* fused decode attention: csrc/cpu/fused_attn_avx2.cpp:145-301         */
/* ------------------------------------------------------------------ */
static void fused_attention_impl(const float* Q, const float* dense_K, const float* dense_V,
                                 int dense_count, const int32_t* PBS_K_Packed,
                                 const void* PBS_K_Scales, const void* PBS_K_Zeroes,
                                 const int32_t* PBS_V_Packed, const void* PBS_V_Scales,
                                 const void* PBS_V_Zeroes, const int64_t* PBS_token_ids,
                                 int num_blocks, int num_q_heads, int num_kv_heads, int head_dim,
                                 float* attn_output, float* mean_attn_weights, int k_group_size,
                                 int meta_fp16, float* logits_out) {
    const float inv_sqrt_hd = 1.0f / sqrtf((float)head_dim);               /* :166 */
    const int total_pbs = num_blocks * k_group_size;
    const int total = dense_count + total_pbs;
    const int gqa = num_kv_heads > 0 ? num_q_heads / num_kv_heads : 1;
    const int words = k_group_size / 16;
    const size_t kvs = (size_t)num_kv_heads * head_dim;
    float* scores = (float*)malloc(sizeof(float) * ((size_t)num_q_heads * total + 1));
    float* kdq = NULL;
    float* vdq = NULL;
    float* row_max = (float*)malloc(sizeof(float) * num_q_heads);
    float* row_sum = (float*)malloc(sizeof(float) * num_q_heads);
    if (num_blocks > 0) {                                                  /* :184-211 */
        kdq = (float*)malloc(sizeof(float) * (size_t)total_pbs * kvs);
        vdq = (float*)malloc(sizeof(float) * (size_t)total_pbs * kvs);
        const size_t meta_bytes = meta_fp16 ? 2 : 4;
        for (int b = 0; b < num_blocks; ++b) {
            orc_dequantize_k(PBS_K_Packed + (size_t)b * words * kvs,
                             (const char*)PBS_K_Scales + (size_t)b * kvs * meta_bytes,
                             (const char*)PBS_K_Zeroes + (size_t)b * kvs * meta_bytes,
                             kdq + (size_t)b * k_group_size * kvs, meta_fp16, 1, num_kv_heads,
                             head_dim, k_group_size);
            orc_dequantize_v(PBS_V_Packed + (size_t)b * k_group_size * num_kv_heads * ((head_dim + 15) / 16),
                             (const char*)PBS_V_Scales + (size_t)b * k_group_size * num_kv_heads * meta_bytes,
                             (const char*)PBS_V_Zeroes + (size_t)b * k_group_size * num_kv_heads * meta_bytes,
                             vdq + (size_t)b * k_group_size * kvs, meta_fp16, k_group_size,
                             num_kv_heads, head_dim);
        }
    }
    for (int h = 0; h < num_q_heads; ++h) {                               /* :222-284 */
        int kv_h = gqa > 1 ? h / gqa : h;
        const float* q = Q + (size_t)h * head_dim;
        float* hs = scores + (size_t)h * total;
        for (int i = 0; i < dense_count; ++i)
            hs[i] = dot8(q, dense_K + ((size_t)i * num_kv_heads + kv_h) * head_dim, head_dim) * inv_sqrt_hd;
        for (int i = 0; i < total_pbs; ++i) {
            if (PBS_token_ids[i] == -1) hs[dense_count + i] = -INFINITY;
            else hs[dense_count + i] = dot8(q, kdq + ((size_t)i * num_kv_heads + kv_h) * head_dim, head_dim) * inv_sqrt_hd;
        }
        float mx = -INFINITY;
        for (int i = 0; i < total; ++i) mx = std_max(mx, hs[i]);
        row_max[h] = mx;
        float sum = 0.0f;
        for (int i = 0; i < total; ++i)
            if (hs[i] != -INFINITY) sum += expf(hs[i] - mx);
        float inv_sum = sum > 0.0f ? (1.0f / sum) : 1.0f;
        row_sum[h] = sum > 0.0f ? sum : 1.0f;
        float* o = attn_output + (size_t)h * head_dim;
        for (int c = 0; c < head_dim; ++c) o[c] = 0.0f;
        for (int i = 0; i < dense_count; ++i) {
            float w = expf(hs[i] - mx) * inv_sum;
            axpy8(o, dense_V + ((size_t)i * num_kv_heads + kv_h) * head_dim, w, head_dim);
        }
        for (int i = 0; i < total_pbs; ++i) {
            if (PBS_token_ids[i] == -1) continue;
            float w = expf(hs[dense_count + i] - mx) * inv_sum;
            axpy8(o, vdq + ((size_t)i * num_kv_heads + kv_h) * head_dim, w, head_dim);
        }
    }
    if (mean_attn_weights) {                                               /* :286-300 */
        for (int i = 0; i < total; ++i) {
            float sw = 0.0f;
            for (int h = 0; h < num_q_heads; ++h) {
                float sc = scores[(size_t)h * total + i];
                if (sc != -INFINITY) sw += expf(sc - row_max[h]) / row_sum[h];
            }
            mean_attn_weights[i] = sw / (float)num_q_heads;
        }
    }
    if (logits_out) memcpy(logits_out, scores, sizeof(float) * (size_t)num_q_heads * total);
    free(scores); free(kdq); free(vdq); free(row_max); free(row_sum);
}

void orc_fused_attention_decode(const float* Q, const float* dense_K, const float* dense_V,
                                int dense_count, const int32_t* PBS_K_Packed,
                                const void* PBS_K_Scales, const void* PBS_K_Zeroes,
                                const int32_t* PBS_V_Packed, const void* PBS_V_Scales,
                                const void* PBS_V_Zeroes, const int64_t* PBS_token_ids,
                                int num_blocks, int num_q_heads, int num_kv_heads, int head_dim,
                                float* attn_output, float* mean_attn_weights, int k_group_size,
                                int meta_fp16) {
    fused_attention_impl(Q, dense_K, dense_V, dense_count, PBS_K_Packed, PBS_K_Scales, PBS_K_Zeroes,
                         PBS_V_Packed, PBS_V_Scales, PBS_V_Zeroes, PBS_token_ids, num_blocks, num_q_heads,
                         num_kv_heads, head_dim, attn_output, mean_attn_weights, k_group_size, meta_fp16, NULL);
}

/* Same computation, also returning the per-head logits s = q.k / sqrt(hd)
 * [num_q_heads][total] (-inf for empty packed slots): lets a test recompute
 * the softmax normalisation in double precision. */
void orc_fused_attention_decode_logits(const float* Q, const float* dense_K, const float* dense_V,
                                       int dense_count, const int32_t* PBS_K_Packed,
                                       const void* PBS_K_Scales, const void* PBS_K_Zeroes,
                                       const int32_t* PBS_V_Packed, const void* PBS_V_Scales,
                                       const void* PBS_V_Zeroes, const int64_t* PBS_token_ids,
                                       int num_blocks, int num_q_heads, int num_kv_heads, int head_dim,
                                       float* attn_output, float* mean_attn_weights, int k_group_size,
                                       int meta_fp16, float* logits) {
    fused_attention_impl(Q, dense_K, dense_V, dense_count, PBS_K_Packed, PBS_K_Scales, PBS_K_Zeroes,
                         PBS_V_Packed, PBS_V_Scales, PBS_V_Zeroes, PBS_token_ids, num_blocks, num_q_heads,
                         num_kv_heads, head_dim, attn_output, mean_attn_weights, k_group_size, meta_fp16, logits);
}

/* ------------------------------------------------------------------ */
/* Engine: csrc/cache_engine.cpp                                       */
/* ------------------------------------------------------------------ */
struct orc_engine {
    orc_engine_params p;
    int chunk, qhd, max_hh;
    size_t kvs;
    int s_count, rw_count, rw_head, hh_count, wr_count;
    int pbs_alloc, pbs_used, pbs_count;
    int total, total_evictions, last_calc_pos;
    float cached_threshold;
    float *S_K, *S_V, *RW_K, *RW_V, *HH_K, *HH_V, *HH_scores, *WR_K, *WR_V;
    int64_t *HH_ids, *WR_ids, *PBS_ids;
    int32_t *PBS_K_Packed, *PBS_V_Packed;
    void *PBS_K_Scales, *PBS_K_Zeroes, *PBS_V_Scales, *PBS_V_Zeroes;
    float* g;
    float *dense_K, *dense_V, *mw;
    size_t mw_cap;
    float* scratch_sel;
};

orc_engine* orc_engine_create(const orc_engine_params* p) {               /* :8-82 */
    orc_engine* e = (orc_engine*)calloc(1, sizeof(orc_engine));
    e->p = *p;
    e->p.k_group_size = (p->k_group_size == 32) ? 32 : 16;
    e->chunk = e->p.k_group_size;
    e->qhd = (p->head_dim + 15) / 16;
    /* std::ceil(max_seq_len * h_ratio): int * float is evaluated in float (:47) */
    e->max_hh = (int)ceilf((float)p->max_seq_len * p->h_ratio);
    if (e->max_hh < 1) e->max_hh = 1;
    e->kvs = (size_t)p->num_kv_heads * p->head_dim;
    e->last_calc_pos = -1;
    e->S_K = (float*)calloc((size_t)p->sink_size * e->kvs + 1, 4);
    e->S_V = (float*)calloc((size_t)p->sink_size * e->kvs + 1, 4);
    e->RW_K = (float*)calloc((size_t)p->rw_size * e->kvs + 1, 4);
    e->RW_V = (float*)calloc((size_t)p->rw_size * e->kvs + 1, 4);
    e->HH_K = (float*)calloc((size_t)e->max_hh * e->kvs, 4);
    e->HH_V = (float*)calloc((size_t)e->max_hh * e->kvs, 4);
    e->HH_ids = (int64_t*)malloc(sizeof(int64_t) * e->max_hh);
    for (int i = 0; i < e->max_hh; ++i) e->HH_ids[i] = -1;
    e->HH_scores = (float*)calloc(e->max_hh, 4);
    e->WR_K = (float*)calloc((size_t)e->chunk * e->kvs, 4);
    e->WR_V = (float*)calloc((size_t)e->chunk * e->kvs, 4);
    e->WR_ids = (int64_t*)malloc(sizeof(int64_t) * e->chunk);
    for (int i = 0; i < e->chunk; ++i) e->WR_ids[i] = -1;
    e->g = (float*)calloc((size_t)p->max_seq_len + 1, 4);
    size_t max_dense = (size_t)p->sink_size + e->max_hh + p->rw_size;
    e->dense_K = (float*)calloc(max_dense * e->kvs + 1, 4);
    e->dense_V = (float*)calloc(max_dense * e->kvs + 1, 4);
    e->mw_cap = max_dense + 1024;
    e->mw = (float*)calloc(e->mw_cap, 4);
    return e;
}

void orc_engine_destroy(orc_engine* e) {
    if (!e) return;
    free(e->S_K); free(e->S_V); free(e->RW_K); free(e->RW_V); free(e->HH_K); free(e->HH_V);
    free(e->HH_ids); free(e->HH_scores); free(e->WR_K); free(e->WR_V); free(e->WR_ids);
    free(e->PBS_K_Packed); free(e->PBS_V_Packed); free(e->PBS_K_Scales); free(e->PBS_K_Zeroes);
    free(e->PBS_V_Scales); free(e->PBS_V_Zeroes); free(e->PBS_ids); free(e->g);
    free(e->dense_K); free(e->dense_V); free(e->mw); free(e->scratch_sel);
    free(e);
}

static void* grow(void* ptr, size_t old_n, size_t new_n, size_t elem) {
    void* q = realloc(ptr, new_n * elem);
    memset((char*)q + old_n * elem, 0, (new_n - old_n) * elem);
    return q;
}

static void ensure_pbs_capacity(orc_engine* e, int min_blocks) {          /* :84-116 */
    if (min_blocks <= e->pbs_alloc) return;
    int nb = e->pbs_alloc + 64 > min_blocks ? e->pbs_alloc + 64 : min_blocks;
    size_t ob = (size_t)e->pbs_alloc;
    size_t words = (size_t)e->p.k_group_size / 16;
    size_t ms = e->p.meta_fp16 ? 2 : 4;
    e->PBS_K_Packed = (int32_t*)grow(e->PBS_K_Packed, ob * words * e->kvs, (size_t)nb * words * e->kvs, 4);
    e->PBS_K_Scales = grow(e->PBS_K_Scales, ob * e->kvs, (size_t)nb * e->kvs, ms);
    e->PBS_K_Zeroes = grow(e->PBS_K_Zeroes, ob * e->kvs, (size_t)nb * e->kvs, ms);
    size_t vm_old = ob * e->chunk * e->p.num_kv_heads, vm_new = (size_t)nb * e->chunk * e->p.num_kv_heads;
    e->PBS_V_Scales = grow(e->PBS_V_Scales, vm_old, vm_new, ms);
    e->PBS_V_Zeroes = grow(e->PBS_V_Zeroes, vm_old, vm_new, ms);
    size_t vps = (size_t)e->p.num_kv_heads * e->qhd;
    e->PBS_V_Packed = (int32_t*)grow(e->PBS_V_Packed, ob * e->chunk * vps, (size_t)nb * e->chunk * vps, 4);
    size_t ids_old = ob * e->chunk, ids_new = (size_t)nb * e->chunk;
    e->PBS_ids = (int64_t*)realloc(e->PBS_ids, ids_new * sizeof(int64_t));
    for (size_t i = ids_old; i < ids_new; ++i) e->PBS_ids[i] = -1;
    e->pbs_alloc = nb;
}

static int cmp_float(const void* a, const void* b) {
    float x = *(const float*)a, y = *(const float*)b;
    return (x > y) - (x < y);
}

static float fetch_or_calc_threshold(orc_engine* e) {                     /* :118-146 */
    int cs = e->p.sink_size, ce = e->total - e->p.rw_size;
    if (ce <= cs) { e->cached_threshold = 0.0f; return 0.0f; }
    if (e->last_calc_pos == -1 || (e->total - e->last_calc_pos >= e->p.update_interval)) {
        size_t n = (size_t)(ce - cs);
        e->scratch_sel = (float*)realloc(e->scratch_sel, n * sizeof(float));
        memcpy(e->scratch_sel, e->g + cs, n * sizeof(float));
        float q = 1.0f - e->p.h_ratio;
        if (q < 0.0f) q = 0.0f;
        if (q > 1.0f) q = 1.0f;
        size_t k = (size_t)(q * (float)(n - 1));
        /* std::nth_element returns the k-th smallest value; any selection
         * algorithm yields the same value. */
        qsort(e->scratch_sel, n, sizeof(float), cmp_float);
        e->cached_threshold = e->scratch_sel[k];
        e->last_calc_pos = e->total;
    }
    return e->cached_threshold;
}

static void flush_wr(orc_engine* e) {                                     /* :148-207 */
    ensure_pbs_capacity(e, e->pbs_used + 1);
    size_t words = (size_t)e->p.k_group_size / 16;
    size_t ms = e->p.meta_fp16 ? 2 : 4;
    size_t b = (size_t)e->pbs_used;
    size_t vps = (size_t)e->p.num_kv_heads * e->qhd;
    orc_quantize_k_block(e->WR_K, (uint32_t*)(e->PBS_K_Packed + b * words * e->kvs),
                         (char*)e->PBS_K_Scales + b * e->kvs * ms, (char*)e->PBS_K_Zeroes + b * e->kvs * ms,
                         e->p.meta_fp16, e->p.num_kv_heads, e->p.head_dim, e->p.k_group_size);
    orc_quantize_v_block(e->WR_V, e->PBS_V_Packed + b * e->chunk * vps,
                         (char*)e->PBS_V_Scales + b * e->chunk * e->p.num_kv_heads * ms,
                         (char*)e->PBS_V_Zeroes + b * e->chunk * e->p.num_kv_heads * ms,
                         e->p.meta_fp16, e->p.num_kv_heads, e->p.head_dim, e->chunk);
    for (int t = 0; t < e->chunk; ++t) e->PBS_ids[b * e->chunk + t] = e->WR_ids[t];
    e->pbs_used++;
    e->pbs_count += e->chunk;
    e->wr_count = 0;
}

static void route(orc_engine* e, const float* k, const float* v, int64_t id) {  /* :209-269 */
    e->total_evictions++;
    size_t kb = e->kvs * sizeof(float);
    float score = (id >= 0 && id < (int64_t)e->p.max_seq_len) ? e->g[id] : 0.0f;
    float thresh = fetch_or_calc_threshold(e);
    if (score >= thresh) {
        if (e->hh_count < e->max_hh) {
            memcpy(e->HH_K + (size_t)e->hh_count * e->kvs, k, kb);
            memcpy(e->HH_V + (size_t)e->hh_count * e->kvs, v, kb);
            e->HH_ids[e->hh_count] = id;
            e->HH_scores[e->hh_count] = score;
            e->hh_count++;
            return;
        }
        int mi = 0;
        float ms = e->HH_scores[0];
        for (int i = 1; i < e->hh_count; ++i)
            if (e->HH_scores[i] < ms) { ms = e->HH_scores[i]; mi = i; }
        if (score > ms) {
            memcpy(e->WR_K + (size_t)e->wr_count * e->kvs, e->HH_K + (size_t)mi * e->kvs, kb);
            memcpy(e->WR_V + (size_t)e->wr_count * e->kvs, e->HH_V + (size_t)mi * e->kvs, kb);
            e->WR_ids[e->wr_count] = e->HH_ids[mi];
            e->wr_count++;
            memcpy(e->HH_K + (size_t)mi * e->kvs, k, kb);
            memcpy(e->HH_V + (size_t)mi * e->kvs, v, kb);
            e->HH_ids[mi] = id;
            e->HH_scores[mi] = score;
            if (e->wr_count == e->chunk) flush_wr(e);
            return;
        }
    }
    memcpy(e->WR_K + (size_t)e->wr_count * e->kvs, k, kb);
    memcpy(e->WR_V + (size_t)e->wr_count * e->kvs, v, kb);
    e->WR_ids[e->wr_count] = id;
    e->wr_count++;
    if (e->wr_count == e->chunk) flush_wr(e);
}

void orc_engine_prefill(orc_engine* e, const float* K_all, const float* V_all, int q_len) {  /* :271-395 */
    size_t kvs = e->kvs, kb = kvs * sizeof(float);
    int S = e->p.sink_size, R = e->p.rw_size;
    if (q_len <= S + R) {
        int s = S < q_len ? S : q_len;
        if (s > 0) {
            memcpy(e->S_K, K_all, (size_t)s * kb);
            memcpy(e->S_V, V_all, (size_t)s * kb);
            e->s_count = s;
        }
        int r = q_len - s;
        if (r > 0) {
            memcpy(e->RW_K, K_all + (size_t)s * kvs, (size_t)r * kb);
            memcpy(e->RW_V, V_all + (size_t)s * kvs, (size_t)r * kb);
            e->rw_count = r;
            e->rw_head = 0;
        }
        e->total = q_len;
        return;
    }
    memcpy(e->S_K, K_all, (size_t)S * kb);
    memcpy(e->S_V, V_all, (size_t)S * kb);
    e->s_count = S;
    int rw_start = q_len - R;
    memcpy(e->RW_K, K_all + (size_t)rw_start * kvs, (size_t)R * kb);
    memcpy(e->RW_V, V_all + (size_t)rw_start * kvs, (size_t)R * kb);
    e->rw_count = R;
    e->rw_head = 0;
    int n_inter = rw_start - S;
    int nblk = n_inter / e->chunk;
    int rem = n_inter % e->chunk;
    if (nblk > 0) {
        ensure_pbs_capacity(e, e->pbs_used + nblk);
        size_t words = (size_t)e->p.k_group_size / 16;
        size_t ms = e->p.meta_fp16 ? 2 : 4;
        size_t vps = (size_t)e->p.num_kv_heads * e->qhd;
        for (int b = 0; b < nblk; ++b) {
            size_t dst = (size_t)e->pbs_used + b;
            int src = S + b * e->chunk;
            orc_quantize_k_block(K_all + (size_t)src * kvs, (uint32_t*)(e->PBS_K_Packed + dst * words * kvs),
                                 (char*)e->PBS_K_Scales + dst * kvs * ms, (char*)e->PBS_K_Zeroes + dst * kvs * ms,
                                 e->p.meta_fp16, e->p.num_kv_heads, e->p.head_dim, e->p.k_group_size);
            orc_quantize_v_block(V_all + (size_t)src * kvs, e->PBS_V_Packed + dst * e->chunk * vps,
                                 (char*)e->PBS_V_Scales + dst * e->chunk * e->p.num_kv_heads * ms,
                                 (char*)e->PBS_V_Zeroes + dst * e->chunk * e->p.num_kv_heads * ms,
                                 e->p.meta_fp16, e->p.num_kv_heads, e->p.head_dim, e->chunk);
            for (int t = 0; t < e->chunk; ++t) e->PBS_ids[dst * e->chunk + t] = src + t;
        }
        e->pbs_used += nblk;
        e->pbs_count += nblk * e->chunk;
        e->total_evictions += nblk * e->chunk;
    }
    if (rem > 0) {
        int rs = S + nblk * e->chunk;
        memcpy(e->WR_K, K_all + (size_t)rs * kvs, (size_t)rem * kb);
        memcpy(e->WR_V, V_all + (size_t)rs * kvs, (size_t)rem * kb);
        for (int t = 0; t < rem; ++t) e->WR_ids[t] = rs + t;
        e->wr_count = rem;
    } else {
        e->wr_count = 0;
    }
    e->total = q_len;
}

void orc_engine_step(orc_engine* e, const float* Q, const float* K_new, const float* V_new,
                     float* attn_output) {                                 /* :397-541 */
    size_t kvs = e->kvs, kb = kvs * sizeof(float);
    int S = e->p.sink_size, R = e->p.rw_size;
    if (e->s_count < S) {
        memcpy(e->S_K + (size_t)e->s_count * kvs, K_new, kb);
        memcpy(e->S_V + (size_t)e->s_count * kvs, V_new, kb);
        e->s_count++;
    } else if (e->rw_count < R) {
        memcpy(e->RW_K + (size_t)e->rw_count * kvs, K_new, kb);
        memcpy(e->RW_V + (size_t)e->rw_count * kvs, V_new, kb);
        e->rw_count++;
    } else {
        int slot = e->rw_head;
        int64_t evicted = (int64_t)e->total - R;
        float* ek = (float*)malloc(kb);
        float* ev = (float*)malloc(kb);
        memcpy(ek, e->RW_K + (size_t)slot * kvs, kb);
        memcpy(ev, e->RW_V + (size_t)slot * kvs, kb);
        memcpy(e->RW_K + (size_t)slot * kvs, K_new, kb);
        memcpy(e->RW_V + (size_t)slot * kvs, V_new, kb);
        e->rw_head = (e->rw_head + 1) % R;
        route(e, ek, ev, evicted);
        free(ek); free(ev);
    }
    e->total++;
    int dc = 0;
    if (e->s_count > 0) {
        memcpy(e->dense_K, e->S_K, (size_t)e->s_count * kb);
        memcpy(e->dense_V, e->S_V, (size_t)e->s_count * kb);
        dc += e->s_count;
    }
    if (e->hh_count > 0) {
        memcpy(e->dense_K + (size_t)dc * kvs, e->HH_K, (size_t)e->hh_count * kb);
        memcpy(e->dense_V + (size_t)dc * kvs, e->HH_V, (size_t)e->hh_count * kb);
        dc += e->hh_count;
    }
    for (int i = 0; i < e->rw_count; ++i) {
        int ri = (e->rw_head + i) % R;
        memcpy(e->dense_K + (size_t)dc * kvs, e->RW_K + (size_t)ri * kvs, kb);
        memcpy(e->dense_V + (size_t)dc * kvs, e->RW_V + (size_t)ri * kvs, kb);
        dc++;
    }
    size_t tt = (size_t)dc + (size_t)e->pbs_used * e->chunk;
    if (e->mw_cap < tt) {
        e->mw = (float*)realloc(e->mw, tt * sizeof(float));
        e->mw_cap = tt;
    }
    orc_fused_attention_decode(Q, e->dense_K, e->dense_V, dc, e->PBS_K_Packed, e->PBS_K_Scales,
                               e->PBS_K_Zeroes, e->PBS_V_Packed, e->PBS_V_Scales, e->PBS_V_Zeroes,
                               e->PBS_ids, e->pbs_used, e->p.num_q_heads, e->p.num_kv_heads,
                               e->p.head_dim, attn_output, e->mw, e->p.k_group_size, e->p.meta_fp16);
    const float d = e->p.score_decay;
    const int msl = e->p.max_seq_len;
    for (int i = 0; i < e->s_count; ++i)
        if (i < msl) e->g[i] = fmaf(d, e->g[i], e->mw[i]);
    for (int i = 0; i < e->hh_count; ++i) {
        int64_t tid = e->HH_ids[i];
        if (tid >= 0 && tid < msl) {
            e->g[tid] = fmaf(d, e->g[tid], e->mw[e->s_count + i]);
            e->HH_scores[i] = e->g[tid];
        }
    }
    int rb = e->total - e->rw_count;
    for (int i = 0; i < e->rw_count; ++i) {
        int tid = rb + i;
        if (tid >= 0 && tid < msl) e->g[tid] = fmaf(d, e->g[tid], e->mw[e->s_count + e->hh_count + i]);
    }
    for (int i = 0; i < e->pbs_used * e->chunk; ++i) {
        int64_t tid = e->PBS_ids[i];
        if (tid >= 0 && tid < msl) e->g[tid] = fmaf(d, e->g[tid], e->mw[dc + i]);
    }
}

size_t orc_engine_buffer_bytes(const orc_engine* e) {                    /* :543-568 */
    size_t ms = e->p.meta_fp16 ? 2 : 4;
    size_t kvs = e->kvs, b = 0;
    size_t words = (size_t)e->p.k_group_size / 16;
    size_t nb = (size_t)e->pbs_alloc;
    b += 2 * (size_t)e->p.sink_size * kvs * 4;
    b += 2 * (size_t)e->p.rw_size * kvs * 4;
    b += 2 * (size_t)e->max_hh * kvs * 4;
    b += (size_t)e->max_hh * 8 + (size_t)e->max_hh * 4;
    b += 2 * (size_t)e->chunk * kvs * 4;
    b += (size_t)e->chunk * 8;
    b += nb * words * kvs * 4;
    b += 2 * nb * kvs * ms + 2 * nb * e->chunk * e->p.num_kv_heads * ms;
    b += nb * e->chunk * e->p.num_kv_heads * e->qhd * 4;
    b += nb * e->chunk * 8;
    b += (size_t)e->p.max_seq_len * 4;
    return b;
}

void orc_engine_counters_get(const orc_engine* e, orc_engine_counters* c) {
    c->s_count = e->s_count;
    c->rw_count = e->rw_count;
    c->rw_head_index = e->rw_head;
    c->hh_count = e->hh_count;
    c->wr_count = e->wr_count;
    c->pbs_allocated_blocks = e->pbs_alloc;
    c->pbs_blocks_used = e->pbs_used;
    c->pbs_count = e->pbs_count;
    c->total_processed_tokens = e->total;
    c->total_evictions = e->total_evictions;
    c->last_calc_pos = e->last_calc_pos;
    c->max_hh = e->max_hh;
    c->chunk_size = e->chunk;
    c->cached_threshold = e->cached_threshold;
}

/* Imports integer state built elsewhere (test infrastructure: synthetic tier
 * layouts written through the buffers); pbs_allocated_blocks and the
 * capacities are not touched. */
void orc_engine_counters_set(orc_engine* e, const orc_engine_counters* c) {
    e->s_count = c->s_count;
    e->rw_count = c->rw_count;
    e->rw_head = c->rw_head_index;
    e->hh_count = c->hh_count;
    e->wr_count = c->wr_count;
    e->pbs_used = c->pbs_blocks_used;
    e->pbs_count = c->pbs_count;
    e->total = c->total_processed_tokens;
    e->total_evictions = c->total_evictions;
    e->last_calc_pos = c->last_calc_pos;
    e->cached_threshold = c->cached_threshold;
}

void* orc_engine_buffer(orc_engine* e, int which, size_t* count, int* elem_size) {
    size_t kvs = e->kvs, nb = (size_t)e->pbs_alloc;
    int ms = e->p.meta_fp16 ? 2 : 4;
    size_t words = (size_t)e->p.k_group_size / 16;
    switch (which) {
    case 0: *count = (size_t)e->p.sink_size * kvs; *elem_size = 4; return e->S_K;
    case 1: *count = (size_t)e->p.sink_size * kvs; *elem_size = 4; return e->S_V;
    case 2: *count = (size_t)e->p.rw_size * kvs; *elem_size = 4; return e->RW_K;
    case 3: *count = (size_t)e->p.rw_size * kvs; *elem_size = 4; return e->RW_V;
    case 4: *count = (size_t)e->max_hh * kvs; *elem_size = 4; return e->HH_K;
    case 5: *count = (size_t)e->max_hh * kvs; *elem_size = 4; return e->HH_V;
    case 6: *count = (size_t)e->max_hh; *elem_size = 8; return e->HH_ids;
    case 7: *count = (size_t)e->max_hh; *elem_size = 4; return e->HH_scores;
    case 8: *count = (size_t)e->chunk * kvs; *elem_size = 4; return e->WR_K;
    case 9: *count = (size_t)e->chunk * kvs; *elem_size = 4; return e->WR_V;
    case 10: *count = (size_t)e->chunk; *elem_size = 8; return e->WR_ids;
    case 11: *count = nb * words * kvs; *elem_size = 4; return e->PBS_K_Packed;
    case 12: *count = nb * kvs; *elem_size = ms; return e->PBS_K_Scales;
    case 13: *count = nb * kvs; *elem_size = ms; return e->PBS_K_Zeroes;
    case 14: *count = nb * e->chunk * e->p.num_kv_heads * e->qhd; *elem_size = 4; return e->PBS_V_Packed;
    case 15: *count = nb * e->chunk * e->p.num_kv_heads; *elem_size = ms; return e->PBS_V_Scales;
    case 16: *count = nb * e->chunk * e->p.num_kv_heads; *elem_size = ms; return e->PBS_V_Zeroes;
    case 17: *count = nb * e->chunk; *elem_size = 8; return e->PBS_ids;
    case 18: *count = (size_t)e->p.max_seq_len; *elem_size = 4; return e->g;
    case 19: *count = e->mw_cap; *elem_size = 4; return e->mw;
    default: *count = 0; *elem_size = 0; return NULL;
    }
}
