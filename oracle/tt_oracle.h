/*
 * tt_oracle.h -- TEST INFRASTRUCTURE ONLY.
 *
 * CPU restatement (plain C, single thread) of TriTierCache's reference
 * algorithms for the decode hot path: K/V 2-bit quantize+pack, dequantize,
 * the fused single-query decode attention and the cache engine
 * (ingest / evict / route / threshold / waiting-room flush / prefill /
 * decayed score feedback).  It is the checker the GPU library is compared
 * against; only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline
 * leg may load it.  The product path never calls it.
 *
 * Parity pin: tests/test_oracle_golden.py checks this restatement against
 * (a) the known-answer vectors of the reference's own C++ tests
 *     (tests/test_quantize_v.cpp, tests/tie_test_v.cpp), and
 * (b) fixtures produced by the reference's own C++ engine and kernels,
 *     compiled from its sources by oracle/Makefile (target `ref`) and dumped
 *     by tests/golden/make_golden.py.
 * The restatement follows the reference's operation order (8-lane FMA dot
 * product tree, sequential softmax sums, glibc expf) so that it reproduces
 * the reference bit for bit on x86-64 with glibc.
 */
#ifndef TT_ORACLE_H
#define TT_ORACLE_H
#include <stdint.h>
#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

/* IEEE binary16 conversions (round to nearest even), as F16C does. */
uint16_t orc_f32_to_f16(float f);
float orc_f16_to_f32(uint16_t h);

/* csrc/cpu/quantize_k_avx2.cpp:26-134 */
void orc_quantize_k_block(const float* K, uint32_t* packed, void* scale_out, void* zero_out,
                          int meta_fp16, int num_heads, int head_dim, int k_group_size);
/* csrc/cpu/quantize_v_avx2.cpp:44-132 */
void orc_quantize_v_block(const float* V, int32_t* packed, void* scale_out, void* zero_out,
                          int meta_fp16, int num_heads, int head_dim, int chunk_size);
/* csrc/cpu/dequantize_avx2.cpp:24-136 */
void orc_dequantize_k(const int32_t* packed, const void* scale, const void* zero, float* out,
                      int meta_fp16, int num_blocks, int num_heads, int head_dim, int k_group_size);
/* csrc/cpu/dequantize_avx2.cpp:138-228 */
void orc_dequantize_v(const int32_t* packed, const void* scale, const void* zero, float* out,
                      int meta_fp16, int total_tokens, int num_heads, int head_dim);

/* csrc/cpu/fused_attn_avx2.cpp:145-357 */
void orc_fused_attention_decode(const float* Q, const float* dense_K, const float* dense_V,
                                int dense_count, const int32_t* PBS_K_Packed,
                                const void* PBS_K_Scales, const void* PBS_K_Zeroes,
                                const int32_t* PBS_V_Packed, const void* PBS_V_Scales,
                                const void* PBS_V_Zeroes, const int64_t* PBS_token_ids,
                                int num_blocks, int num_q_heads, int num_kv_heads, int head_dim,
                                float* attn_output, float* mean_attn_weights, int k_group_size,
                                int meta_fp16);

/* the same, also writing the per-head logits [num_q_heads][total] */
void orc_fused_attention_decode_logits(const float* Q, const float* dense_K, const float* dense_V,
                                       int dense_count, const int32_t* PBS_K_Packed,
                                       const void* PBS_K_Scales, const void* PBS_K_Zeroes,
                                       const int32_t* PBS_V_Packed, const void* PBS_V_Scales,
                                       const void* PBS_V_Zeroes, const int64_t* PBS_token_ids,
                                       int num_blocks, int num_q_heads, int num_kv_heads, int head_dim,
                                       float* attn_output, float* mean_attn_weights, int k_group_size,
                                       int meta_fp16, float* logits);

/* csrc/include/cache_engine.h:10-123 */
typedef struct orc_engine orc_engine;

typedef struct {
    int num_q_heads, num_kv_heads, head_dim, max_seq_len;
    int sink_size, rw_size;
    float h_ratio, score_decay;
    int update_interval, k_group_size, meta_fp16;
} orc_engine_params;

typedef struct {
    int s_count, rw_count, rw_head_index, hh_count, wr_count;
    int pbs_allocated_blocks, pbs_blocks_used, pbs_count;
    int total_processed_tokens, total_evictions, last_calc_pos, max_hh, chunk_size;
    float cached_threshold;
} orc_engine_counters;

/* cache_engine.cpp:8-82 (k_group_size coerced to 16 unless 32, :29) */
orc_engine* orc_engine_create(const orc_engine_params* p);
void orc_engine_destroy(orc_engine* e);
/* cache_engine.cpp:397-541 */
void orc_engine_step(orc_engine* e, const float* Q, const float* K_new, const float* V_new,
                     float* attn_output);
/* cache_engine.cpp:271-395 */
void orc_engine_prefill(orc_engine* e, const float* K_all, const float* V_all, int q_len);
/* cache_engine.cpp:543-568 */
size_t orc_engine_buffer_bytes(const orc_engine* e);
void orc_engine_counters_get(const orc_engine* e, orc_engine_counters* c);
/* test infrastructure: overwrite the integer state (not the capacities) */
void orc_engine_counters_set(orc_engine* e, const orc_engine_counters* c);

/* Raw buffer access (the reference exposes the same buffers as writable
 * zero-copy views, bindings.cpp:461-626).  which: 0 S_K, 1 S_V, 2 RW_K,
 * 3 RW_V, 4 HH_K, 5 HH_V, 6 HH_token_ids, 7 HH_scores, 8 WR_K, 9 WR_V,
 * 10 WR_token_ids, 11 PBS_K_Packed, 12 PBS_K_Scales, 13 PBS_K_Zeroes,
 * 14 PBS_V_Packed, 15 PBS_V_Scales, 16 PBS_V_Zeroes, 17 PBS_token_ids,
 * 18 global_attn_scores, 19 mean_attn_weights (last step).
 * Returns the pointer and writes the element count and element size. */
void* orc_engine_buffer(orc_engine* e, int which, size_t* count, int* elem_size);

#ifdef __cplusplus
}
#endif
#endif
