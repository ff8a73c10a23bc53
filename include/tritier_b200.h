/*
 * tritier_b200.h -- C ABI of the B200 (sm_100a) TriTierCache decode library
 * (libtritier_b200.so).
 *
 * Every pointer argument is a DEVICE pointer (cudaMalloc / torch CUDA tensor
 * memory) unless stated otherwise.  `stream` is a cudaStream_t passed as
 * void* (NULL = legacy default stream).  Calls are stream-ordered and do not
 * synchronise the device unless stated.  Every entry point returns a
 * tt_status; the message of the last failure on the calling thread is
 * available from tt_last_error().  No C++ exception crosses this boundary.
 *
 * Metadata ("pbs_metadata_dtype"): meta_fp16 = 1 selects IEEE binary16
 * scale/zero stored as raw uint16 bits, 0 selects float32 -- the two storage
 * formats of the reference (csrc/include/quantize_k_avx2.h:5-24).
 *
 * Each declaration names the reference interface it replaces (paths relative
 * to the reference project root).
 */
#ifndef TRITIER_B200_H
#define TRITIER_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#pragma GCC visibility push(default)
#endif

typedef enum {
    TT_OK = 0,
    TT_ERR_INVALID_ARGUMENT = 1, /* reference std::invalid_argument -> ValueError (bindings.cpp:324) */
    TT_ERR_OUT_OF_RANGE = 2,     /* reference std::out_of_range -> IndexError (bindings.cpp:326) */
    TT_ERR_OUT_OF_MEMORY = 3,    /* reference std::bad_alloc -> MemoryError (bindings.cpp:328) */
    TT_ERR_CUDA = 4,             /* CUDA runtime failure -> RuntimeError */
    TT_ERR_TIMEOUT = 5,          /* a bounded device-side wait gave up -> RuntimeError */
    TT_ERR_UNSUPPORTED = 6       /* shape outside what the kernels are built for -> ValueError */
} tt_status;

/* Message of the last failing call on this thread ("" if none). */
const char* tt_last_error(void);
/* Library version string and the compute capability the kernels target. */
const char* tt_version(void);
/* 1 when `p` is device (or managed) memory the kernels can dereference, 0
 * otherwise.  Lets a binding accept raw integer addresses the way the
 * reference's get_contiguous_ptr does (bindings.cpp:34-44) and stage host
 * buffers through the device.  No compute. */
int tt_pointer_is_device(const void* p);

/* Kernel timing for benchmarks.  While enabled, every kernel launch of the
 * library is bracketed by CUDA events recorded on its own stream;
 * tt_profile_collect() waits for them, returns the summed durations per
 * kernel kind and clears the record.  Off by default; no reference
 * counterpart. */
typedef struct {
    double maintain_ms;   /* k_engine_maintain */
    double partial_ms;    /* the attention kernels, dense and packed, fork to join (dominant) */
    double finalize_ms;   /* k_attn_finalize */
    int maintain_launches, partial_launches, finalize_launches;
} tt_kernel_times;
tt_status tt_profile_enable(int on);
tt_status tt_profile_collect(tt_kernel_times* out);

/* Synchronises the device and reports the first device-side error recorded by
 * the library's kernels (a bounded wait that expired: TT_ERR_TIMEOUT), 0 if
 * none; clear != 0 resets it.  No reference counterpart. */
tt_status tt_device_error(int clear, int* out);

/* ---------------------------------------------------------------------- */
/* Stand-alone kernels                                                     */
/* ---------------------------------------------------------------------- */

/* Fused single-query decode attention over a dense FP32 token set and the
 * 2-bit packed background store.  Replaces fused_attention_decode_avx2
 * (csrc/include/fused_attn_avx2.h:4-40; binding bindings.cpp:99-178,
 * :340-363).  Layouts (row-major):
 *   Q [num_q_heads, head_dim]; dense_K/V [dense_count, num_kv_heads, head_dim];
 *   PBS_K_Packed [num_blocks*(k_group_size/16), num_kv_heads, head_dim] int32;
 *   PBS_K_Scales/Zeroes [num_blocks, num_kv_heads, head_dim];
 *   PBS_V_Packed [num_blocks*k_group_size, num_kv_heads, ceil(head_dim/16)];
 *   PBS_V_Scales/Zeroes [num_blocks*k_group_size, num_kv_heads];
 *   PBS_token_ids [num_blocks*k_group_size] int64, -1 = empty slot (excluded);
 *   attn_output [num_q_heads, head_dim];
 *   mean_attn_weights [dense_count + num_blocks*k_group_size] or NULL.
 * Dense/PBS pointers may be NULL when their count is 0.  Negative counts ->
 * TT_ERR_INVALID_ARGUMENT (bindings.cpp:120-128).  Scratch comes from a
 * per-device workspace owned by the library (grown on demand). */
tt_status tt_fused_attention_decode(
    const float* Q, const float* dense_K, const float* dense_V, int dense_count,
    const int32_t* PBS_K_Packed, const void* PBS_K_Scales, const void* PBS_K_Zeroes,
    const int32_t* PBS_V_Packed, const void* PBS_V_Scales, const void* PBS_V_Zeroes,
    const int64_t* PBS_token_ids, int num_blocks, int num_q_heads, int num_kv_heads,
    int head_dim, float* attn_output, float* mean_attn_weights, int k_group_size,
    int meta_fp16, void* stream);

/* Same arguments, layouts and results as tt_fused_attention_decode, but the
 * call allocates nothing: its scratch is a fixed 32 MiB array in device
 * memory, declared at file scope in the library, instead of a workspace grown
 * with cudaMalloc.  It is for callers that must not allocate device memory
 * after start-up (a process that reserves the GPU's memory up front, a host
 * framework whose allocator owns device memory, a loop where cudaMalloc's
 * possible device synchronisation is not acceptable).  Calls whose scratch
 * need (partials of every split-KV chunk plus num_q_heads x tokens logits)
 * exceeds 32 MiB return TT_ERR_INVALID_ARGUMENT with a message.  Every call
 * on a device shares the one array and leaves its contents behind, so calls
 * that overlap on the GPU (different streams, or threads) race; keep them
 * ordered.  The first call on a device looks up the array's device address
 * (cudaGetSymbolAddress).  With CUDA's default lazy module loading that
 * lookup is also what loads the module holding the array, so the first call
 * on each device reserves the 32 MiB; make it at start-up, before reserving
 * the device's memory and before any stream capture (or set
 * CUDA_MODULE_LOADING=EAGER).  From then on the device holds the array until
 * the process exits.  The address is cached per device for the life of the
 * process; do not call this entry point again after a cudaDeviceReset.
 * No counterpart in the reference (its CPU kernel keeps thread-local scratch
 * vectors, fused_attn_avx2.cpp:139-143). */
tt_status tt_fused_attention_decode_noalloc(
    const float* Q, const float* dense_K, const float* dense_V, int dense_count,
    const int32_t* PBS_K_Packed, const void* PBS_K_Scales, const void* PBS_K_Zeroes,
    const int32_t* PBS_V_Packed, const void* PBS_V_Scales, const void* PBS_V_Zeroes,
    const int64_t* PBS_token_ids, int num_blocks, int num_q_heads, int num_kv_heads,
    int head_dim, float* attn_output, float* mean_attn_weights, int k_group_size,
    int meta_fp16, void* stream);

/* One K block: K [k_group_size, num_heads, head_dim] -> packed
 * [k_group_size/16, num_heads, head_dim] words, scale/zero [num_heads, head_dim].
 * Bit-exact with quantize_k_block_avx2 (csrc/include/quantize_k_avx2.h:4-20;
 * binding bindings.cpp:180-212). */
tt_status tt_quantize_k_block(const float* K, uint32_t* packed, void* scale, void* zero,
                              int num_heads, int head_dim, int k_group_size, int meta_fp16,
                              void* stream);

/* One V chunk: V [chunk_size, num_heads, head_dim] -> packed
 * [chunk_size, num_heads, ceil(head_dim/16)] words, scale/zero
 * [chunk_size, num_heads].  Bit-exact with quantize_v_block_avx2
 * (csrc/include/quantize_v_avx2.h:4-19; binding bindings.cpp:214-246).
 * head_dim must be a multiple of 16 (the reference reads past the row
 * otherwise, csrc/cpu/quantize_v_avx2.cpp:91-92). */
tt_status tt_quantize_v_block(const float* V, int32_t* packed, void* scale, void* zero,
                              int num_heads, int head_dim, int chunk_size, int meta_fp16,
                              void* stream);

/* Replaces dequantize_k_avx2 (csrc/include/dequant_avx2.h:4-21; binding
 * bindings.cpp:248-281): out [num_blocks*k_group_size, num_heads, head_dim]. */
tt_status tt_dequantize_k(const int32_t* packed, const void* scale, const void* zero,
                          float* out, int num_blocks, int num_heads, int head_dim,
                          int k_group_size, int meta_fp16, void* stream);

/* Replaces dequantize_v_avx2 (csrc/include/dequant_avx2.h:23-38; binding
 * bindings.cpp:283-315): out [total_tokens, num_heads, head_dim]. */
tt_status tt_dequantize_v(const int32_t* packed, const void* scale, const void* zero,
                          float* out, int total_tokens, int num_heads, int head_dim,
                          int meta_fp16, void* stream);

/* ---------------------------------------------------------------------- */
/* Cache engine (device-resident tier state)                              */
/* ---------------------------------------------------------------------- */

/* Constructor arguments of TriTierCacheEngine (csrc/include/cache_engine.h:81-93;
 * binding bindings.cpp:385-398).  k_group_size is coerced to 16 unless 32
 * (cache_engine.cpp:29).  device = CUDA ordinal that owns the state. */
typedef struct {
    int num_q_heads;
    int num_kv_heads;
    int head_dim;
    int max_seq_len;
    int sink_size;
    int rw_size;
    float h_ratio;
    float score_decay;
    int update_interval;
    int k_group_size;
    int meta_fp16;
    int device;
} tt_engine_config;

typedef struct tt_engine tt_engine;

/* Counters exposed read-only by the reference binding (bindings.cpp:437-458)
 * plus the waiting-room fill and the cached threshold. */
typedef struct {
    int s_count, rw_count, rw_head_index, hh_count, wr_count;
    int pbs_allocated_blocks, pbs_blocks_used, pbs_count;
    int total_processed_tokens, total_evictions, last_calc_pos, max_hh, chunk_size;
    float cached_threshold;
} tt_engine_counters;

/* Buffer identifiers for tt_engine_get_buffer (the zero-copy views of
 * bindings.cpp:461-626, plus the waiting room). */
typedef enum {
    TT_BUF_S_K = 0, TT_BUF_S_V, TT_BUF_RW_K, TT_BUF_RW_V, TT_BUF_HH_K, TT_BUF_HH_V,
    TT_BUF_HH_TOKEN_IDS, TT_BUF_HH_SCORES, TT_BUF_WR_K, TT_BUF_WR_V, TT_BUF_WR_TOKEN_IDS,
    TT_BUF_PBS_K_PACKED, TT_BUF_PBS_K_SCALES, TT_BUF_PBS_K_ZEROES, TT_BUF_PBS_V_PACKED,
    TT_BUF_PBS_V_SCALES, TT_BUF_PBS_V_ZEROES, TT_BUF_PBS_TOKEN_IDS, TT_BUF_GLOBAL_ATTN_SCORES,
    TT_BUF_COUNT
} tt_buffer_id;

typedef struct {
    void* data;        /* device pointer */
    size_t count;      /* elements visible to the reference view */
    int elem_size;     /* bytes per element */
    int dtype;         /* 0 float32, 1 int32, 2 int64, 3 uint16 (binary16 bits) */
} tt_buffer_desc;

/* Replaces TriTierCacheEngine::TriTierCacheEngine (cache_engine.cpp:8-82). */
tt_status tt_engine_create(const tt_engine_config* cfg, tt_engine** out);
tt_status tt_engine_destroy(tt_engine* e);

/* Replaces TriTierCacheEngine::step (cache_engine.cpp:397-541; binding
 * bindings.cpp:399-417): ingest one token (K_new/V_new [num_kv_heads*head_dim]),
 * evict/route/flush, attend with Q [num_q_heads*head_dim] into attn_output,
 * decayed score feedback.  Stream-ordered, no host synchronisation. */
tt_status tt_engine_step(tt_engine* e, const float* Q, const float* K_new, const float* V_new,
                         float* attn_output, void* stream);

/* One decode step for n independent engines (layers and/or sequences) in one
 * set of launches.  Q/K_new/V_new/attn_output are host arrays of n device
 * pointers.  All engines must live on the same device.  No reference
 * counterpart: the reference is batch-1, one engine per call
 * (src/tri_tier/integration/patch_model.py:65). */
tt_status tt_engine_step_batched(tt_engine* const* engines, int n, const float* const* Q,
                                 const float* const* K_new, const float* const* V_new,
                                 float* const* attn_output, void* stream);

/* Sequence-sharded decode step over `world` GPUs (one process per GPU).
 * Every rank holds the same engines (same configuration, same inputs every
 * step, so the same tier contents).  Each token has one owner rank while it
 * stays in a tier slot: sink, heavy-hitter and ring slot j belong to rank
 * j % world, packed tokens to ranks in granules of 256 (granule k to rank
 * k % world).  A rank attends only the tokens it owns and alone keeps their
 * accumulated scores current.  Attention over a token set merges exactly
 * through (max, sum, weighted sum) rows, the decomposition the reference's
 * softmax (fused_attn_avx2.cpp:245-284) allows; the reference itself has no
 * multi-GPU path.  One step is two calls, stream-ordered, around two
 * all-gathers the caller performs with its collective library (NCCL, MPI,
 * ...), all ranks in the same order:
 *
 *   tt_engine_step_sharded_begin(..., route_all, xch_send)
 *       maintenance (routing from route_all) + partial attention;
 *       xch_send: n * num_q_heads * (head_dim + 2) floats (device)
 *   all-gather xch_send -> xch_all [world][n][num_q_heads][head_dim + 2]
 *       (xch_all 8-byte aligned, else TT_ERR_INVALID_ARGUMENT)
 *   tt_engine_step_sharded_merge(..., xch_all, attn_output, route_send)
 *       attn_output identical on every rank; score feedback of this rank's
 *       tokens; route_send: n routing rows of 16 bytes (device, 16-byte
 *       aligned): the score of the token the next step evicts (from the
 *       owner of its ring slot) and this rank's smallest heavy-hitter
 *       (score, slot)
 *   all-gather route_send -> route_all [world][n] rows, for the next begin.
 *
 * route_all = NULL routes from the rank's own scores, which is right when
 * every rank holds every token's current score: after prefill, after steps
 * that were not sharded, and after a score synchronisation.  Every
 * update_interval tokens the maintenance recomputes the heavy-hitter
 * threshold, a percentile over all scores (cache_engine.cpp:118-146); before
 * such a step (tt_engine_sharded_sync_needed sets *need) the caller
 * synchronises the scores and passes route_all = NULL (begin refuses a
 * route_all then, with TT_ERR_INVALID_ARGUMENT):
 *
 *   tt_engine_sharded_scores_floats(engines, n, &f)       (host only)
 *   tt_engine_sharded_scores_pack(..., buf)   buf[f]: the owned scores, zeros elsewhere
 *   all-reduce (sum) buf over the ranks       exact: one nonzero term per token
 *   tt_engine_sharded_scores_unpack(..., buf) every score current on every rank
 *
 * n <= 64, world <= 64.  A rank that skips a call leaves its engines out of
 * step with the others. */
tt_status tt_engine_step_sharded_begin(tt_engine* const* engines, int n, const float* const* Q,
                                       const float* const* K_new, const float* const* V_new, int rank,
                                       int world, const void* route_all, float* xch_send, void* stream);
tt_status tt_engine_step_sharded_merge(tt_engine* const* engines, int n, int rank, int world,
                                       const float* xch_all, float* const* attn_output, void* route_send,
                                       void* stream);
tt_status tt_engine_sharded_sync_needed(tt_engine* const* engines, int n, int* need);
tt_status tt_engine_sharded_scores_floats(tt_engine* const* engines, int n, long long* floats);
tt_status tt_engine_sharded_scores_pack(tt_engine* const* engines, int n, int rank, int world, float* buf,
                                        void* stream);
tt_status tt_engine_sharded_scores_unpack(tt_engine* const* engines, int n, const float* buf, void* stream);

/* The same sharded step with the two per-step exchanges done by the library
 * itself over NVLink peer memory (CUDA IPC) instead of by the caller's
 * collectives: every rank owns an exchange region that all ranks write
 * into, and the kernels wait for the other ranks' rows with bounded spins on
 * step-numbered flags (a wait that runs out records TT_ERR_TIMEOUT in the
 * engines' error word, reported by tt_engine_get_counters).  For the ranks of
 * one node (2..8), one process per GPU:
 *
 *   tt_sharded_xch_create(world, rank, n, nq, hd, device, &x, handle)
 *       handle: 64 bytes out (a CUDA IPC handle of this rank's region)
 *   all-gather the handles in rank order (world * 64 bytes)
 *   tt_sharded_xch_open(x, handles)
 *   per step: [score synchronisation as above when needed, then route_valid = 0]
 *       tt_engine_step_sharded_begin_xch(..., x, route_valid, stream)
 *       tt_engine_step_sharded_merge_xch(..., x, attn_output, stream)
 *   all ranks finished every step (e.g. a barrier), then tt_sharded_xch_destroy(x)
 *
 * route_valid = 0 on the first step and after a score synchronisation (the
 * same rule as route_all = NULL above); every rank makes the same calls. */
typedef struct tt_xch tt_xch;
tt_status tt_sharded_xch_create(int world, int rank, int max_engines, int num_q_heads, int head_dim, int device,
                                tt_xch** out, void* ipc_handle);
tt_status tt_sharded_xch_open(tt_xch* x, const void* ipc_handles);
tt_status tt_sharded_xch_destroy(tt_xch* x);
tt_status tt_engine_step_sharded_begin_xch(tt_engine* const* engines, int n, const float* const* Q,
                                           const float* const* K_new, const float* const* V_new, tt_xch* x,
                                           int route_valid, void* stream);
tt_status tt_engine_step_sharded_merge_xch(tt_engine* const* engines, int n, tt_xch* x,
                                           float* const* attn_output, void* stream);

/* Replaces TriTierCacheEngine::prefill (cache_engine.cpp:271-395; binding
 * bindings.cpp:418-436): K_all/V_all [q_len, num_kv_heads, head_dim].
 * q_len < 0 -> TT_ERR_INVALID_ARGUMENT. */
tt_status tt_engine_prefill(tt_engine* e, const float* K_all, const float* V_all, int q_len,
                            void* stream);

/* The per-token half of the reference's full-weights decode path
 * (output_attentions=True, src/tri_tier/integration/patch_model.py:163-169):
 *
 * tt_engine_ingest replaces TriTierCache.ingest_token (src/tri_tier/cache.py:
 * 206-233): the new token K_new/V_new [num_kv_heads*head_dim] enters the sink
 * / ring tiers and the evicted ring token is routed and, with a full waiting
 * room, quantized -- the engine's own maintenance (cache_engine.cpp:405-431,
 * :209-269), without attention and without score feedback.  Stream-ordered. */
tt_status tt_engine_ingest(tt_engine* e, const float* K_new, const float* V_new, void* stream);

/* Number of positions tt_engine_reconstruct returns: sinks + heavy hitters +
 * live packed tokens + ring.  Synchronises. */
tt_status tt_engine_full_count(tt_engine* e, int* count);

/* Replaces TriTierCache.reconstruct_full_cache (src/tri_tier/cache.py:326-372):
 * K_out/V_out [capacity, num_kv_heads, head_dim] float32 and ids_out
 * [capacity] int64 receive the rows [sinks | heavy hitters and live packed
 * tokens in token-id order | ring in logical order], packed tokens
 * dequantized as code*scale + zero (two roundings, as the reference's torch
 * expression).  *count = rows written; capacity below it ->
 * TT_ERR_INVALID_ARGUMENT (nothing written).  Synchronises. */
tt_status tt_engine_reconstruct(tt_engine* e, float* K_out, float* V_out, int64_t* ids_out, int capacity,
                                int* count, void* stream);

/* Replaces TriTierCache.accumulate_attn_scrs (src/tri_tier/cache.py:164-187):
 * global_attn_scores[ids[i]] += mean over heads of weights[h][i] for every
 * i < n with ids[i] in [0, max_seq_len) (undecayed; ids NULL means ids[i] = i).
 * weights [n_heads, n] float32.  Stream-ordered. */
tt_status tt_engine_accumulate_scores(tt_engine* e, const float* weights, const int64_t* ids, int n_heads, int n,
                                      void* stream);

/* Reads the device-side counters (synchronises the engine's last stream). */
tt_status tt_engine_get_counters(tt_engine* e, tt_engine_counters* out);

/* Overwrites the engine's integer state (all fields of `c` except max_hh and
 * chunk_size), stream-ordered on `stream`.  Together with the writable
 * buffers of tt_engine_get_buffer this imports a tier layout built elsewhere
 * (synthetic benchmark states, checkpoints).  The caller keeps the state
 * consistent (counts within capacity, ids of the packed blocks written).
 * No reference counterpart: the reference exposes its counters read-only
 * (bindings.cpp:437-458). */
tt_status tt_engine_set_counters(tt_engine* e, const tt_engine_counters* c, void* stream);

/* Device pointer and reference-view extent of one tier buffer.  PBS views
 * are sized by pbs_allocated_blocks (bindings.cpp:545-626); the pointer
 * stays valid until the engine's PBS storage grows. */
tt_status tt_engine_get_buffer(tt_engine* e, int which, tt_buffer_desc* out);

/* Replaces TriTierCacheEngine::get_buffer_bytes (cache_engine.cpp:543-568):
 * the reference's byte formula over its logical buffer sizes. */
tt_status tt_engine_get_buffer_bytes(tt_engine* e, size_t* out);

/* Bytes this engine actually holds on the device (tiers, PBS capacity,
 * attention scratch).  No reference counterpart. */
tt_status tt_engine_device_bytes(tt_engine* e, size_t* out);

#if defined(__GNUC__)
#pragma GCC visibility pop
#endif

#ifdef __cplusplus
}
#endif
#endif /* TRITIER_B200_H */
