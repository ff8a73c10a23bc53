// tt_attn.cuh -- job description shared by the fused decode attention
// kernels (tt_attn.cu) and the cache engine (tt_engine.cu).
#pragma once
#include "tt_common.cuh"

namespace tt {

// Device-resident counters of one engine (authoritative tier state; the
// reference keeps the same integers as members, csrc/include/cache_engine.h).
struct DevCounters {
    int s_count, rw_count, rw_head, hh_count, wr_count;
    int pbs_alloc, pbs_used, pbs_count;
    int total, total_evictions, last_calc_pos;
    float cached_threshold;
    int error;     // sticky device-side error code (tt_status), 0 = none
    int pad[3];
};

// Everything one attention job reads and writes.  For an engine the tier
// counts come from `ctr` (written by the maintenance kernel earlier on the
// same stream); for the stand-alone call they are the static fields.
// Logical token order (the order of mean_attn_weights, fused_attn_avx2.cpp:
// 228-245 and cache_engine.cpp:433-459): [seg0 | seg1 | seg2 (ring) | PBS].
struct JobDesc {
    int nq, nkv, hd, grp, meta16;
    int n0, n1, n2, ring_head, ring_size, nblk;  // static counts (ctr == nullptr)
    const float *K0, *V0, *K1, *V1, *K2, *V2;    // sinks | heavy hitters | recent ring
    const int32_t* kp;
    const void* ks;
    const void* kz;
    const int32_t* vp;
    const void* vs;
    const void* vz;
    const int64_t* ids;
    const DevCounters* ctr;
    // scratch
    float* part_ml;   // [max_chunks][nq][2]  (m in log2 units, l)
    float* part_acc;  // [max_chunks][nq][hd]
    float* scores;    // [nq][score_stride]  (log2-domain logits)
    int score_stride;
    int max_chunks;
    // score feedback (engine only)
    float* g;                  // global_attn_scores [msl]
    float* hh_scores;          // HH_scores [max_hh]
    const int64_t* hh_ids;     // HH_token_ids
    float decay;
    int msl;
};

struct TierCounts {
    int n0, n1, n2, ring_head, ring_size, nblk, total;
};

__device__ __forceinline__ TierCounts resolve_counts(const JobDesc& j) {
    TierCounts t;
    if (j.ctr) {
        const volatile DevCounters* c = j.ctr;
        t.n0 = c->s_count;
        t.n1 = c->hh_count;
        t.n2 = c->rw_count;
        t.ring_head = c->rw_head;
        t.nblk = c->pbs_used;
        t.total = c->total;
    } else {
        t.n0 = j.n0;
        t.n1 = j.n1;
        t.n2 = j.n2;
        t.ring_head = j.ring_head;
        t.nblk = j.nblk;
        t.total = 0;
    }
    t.ring_size = j.ring_size;
    return t;
}

// Host-side launch description.
constexpr int kMaxBatch = 64;

struct AttnLaunch {
    int njobs;
    int nhg;      // kv-head groups per job (grid.y = njobs * nhg)
    int HG;       // kv heads per group (1, 2, 4 or 8)
    int G;        // q heads per kv head
    int nd;       // dense chunk slots per job (grid.x = nd + np)
    int np;       // PBS chunk slots per job
    int DC;       // dense tokens per chunk (multiple of 32)
    int PC;       // PBS tokens per chunk (multiple of 32)
    int meta_bytes;  // largest PBS metadata element of the batch (2 or 4): sizes the staging buffers
    int rank, world; // sequence sharding: this launch attends only its share (world <= 1: everything)
    // merge_mode: the last partial CTA of each job merges the job's chunks
    // (0 no: separate merge kernel; 1 -> out + (M, 1/L); 2 -> xch rows).  Callers
    // set 1 to allow it (only engines: their per-job arrival counters start at
    // zero); the launch functions pick the mode per launch.
    int merge_mode;
    float* xch;      // merge_mode 2: [njobs][nq][hd + 2] (m, l, acc) rows
    const JobDesc* jobs[kMaxBatch];  // device descriptor per job (engines) or nullptr
    JobDesc inline_job;              // stand-alone job (jobs[0] == nullptr, njobs == 1)
    const float* Q[kMaxBatch];
    float* out[kMaxBatch];
    float* mw[kMaxBatch];     // mean_attn_weights output (stand-alone) or nullptr
};

// Picks chunk sizes and grid extents for `njobs` jobs whose largest token
// capacities are dense_cap / pbs_tok_cap.  Returns TT_ERR_UNSUPPORTED for
// shapes the kernels are not built for.
tt_status plan_attention(AttnLaunch& L, int nq, int nkv, int hd, int dense_cap, int pbs_tok_cap);

// The tokens one rank of `world` attends: dense positions [dlo, dhi) and
// packed token offsets [plo, phi) (whole blocks).  Every rank derives the same
// split from the same (replicated) counters.
struct ShardRange {
    int dlo, dhi, plo, phi;
};
__host__ __device__ __forceinline__ ShardRange shard_range(int D, int nblk, int grp, int rank, int world) {
    ShardRange r;
    if (world <= 1) {
        r.dlo = 0; r.dhi = D; r.plo = 0; r.phi = nblk * grp;
    } else {
        r.dlo = (int)((long long)D * rank / world);
        r.dhi = (int)((long long)D * (rank + 1) / world);
        r.plo = (int)((long long)nblk * rank / world) * grp;
        r.phi = (int)((long long)nblk * (rank + 1) / world) * grp;
    }
    return r;
}
// Scratch a job needs for a given plan: chunk slots and score stride.
int attn_max_chunks(int dense_cap, int pbs_tok_cap);
// Launches the partial, head-merge and weights kernels on `stream`.
tt_status launch_attention(const AttnLaunch& L, cudaStream_t stream);

// Sequence-sharded attention, three stream-ordered phases around two
// all-gathers done by the caller (L.rank / L.world set, L.mw unused):
//  1. partial attention over this rank's share, merged into one
//     (m, l, acc[hd]) row per (job, head): xch[job][h][hd + 2];
//  2. given every rank's rows (xch_all[world][njobs][nq][hd + 2]): the output
//     (same arithmetic and order on every rank) and the mean attention weights
//     of this rank's positions: mw_send[job][slot_cap];
//  3. given every rank's weights (mw_all[world][njobs][slot_cap]): score
//     feedback for all positions, identical on every rank.
tt_status launch_sharded_partial(const AttnLaunch& L, float* xch, cudaStream_t stream);
tt_status launch_sharded_merge(const AttnLaunch& L, const float* xch_all, float* mw_send, int slot_cap,
                               cudaStream_t stream);
tt_status launch_sharded_feedback(const AttnLaunch& L, const float* mw_all, int slot_cap, cudaStream_t stream);

}  // namespace tt
