// tt_attn.cuh -- job description shared by the fused decode attention
// kernels (tt_attn.cu) and the cache engine (tt_engine.cu).
#pragma once
#include <string.h>

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

// Peer-memory exchange of a sequence-sharded step (one node, CUDA IPC over
// NVLink; world > 1 enables it).  Every rank owns a region that all ranks
// write into: rows [world][jobs][nq][hd + 2] floats, routing rows
// [world][jobs] and flags [2][world][jobs] (u64): flag[0][p][j] is the last
// step whose exchange rows rank p has published for job j, flag[1][p][j] the
// same for its routing row.  rows[p] / route[p] / flags[p] are rank p's region
// as this rank addresses it (its own for p == rank).
constexpr int kMaxWorld = 8;
struct PeerXch {
    int world, rank, jobs;  // jobs: the regions' job capacity (stride of the rank slots)
    long long step;         // the step being run (flags start at 0, steps at 1)
    float* rows[kMaxWorld];
    void* route[kMaxWorld];
    unsigned long long* flags[kMaxWorld];
};

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
    PeerXch px;      // merge_mode 2 with px.world > 1: the rows go to every rank's region
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

// Sequence sharding over `world` ranks.  Every token has one owner rank for
// as long as it stays in one tier slot: sink, heavy-hitter and ring slot j
// belong to rank j mod world, the packed tier to ranks in granules of
// kShardGran tokens (granule k to rank k mod world).  A rank attends exactly
// the tokens it owns and alone keeps their accumulated scores up to date, so
// the ranks need not exchange per-position weights.  A rank's positions are
// numbered locally: its dense positions first (its sinks, then its heavy
// hitters, then its ring slots, in slot order), then its packed tokens in
// granule order.  world <= 1: local = global numbering.
constexpr int kShardGran = 256;

__host__ __device__ __forceinline__ int owned_count(int n, int r, int w) { return n > r ? (n - r + w - 1) / w : 0; }

struct ShardMap {
    int nd, np;  // this rank's dense positions and packed tokens
};
__host__ __device__ __forceinline__ ShardMap shard_map(const TierCounts& tc, int grp, int r, int w) {
    ShardMap m;
    const int P = tc.nblk * grp;
    if (w <= 1) {
        m.nd = tc.n0 + tc.n1 + tc.n2;
        m.np = P;
        return m;
    }
    m.nd = owned_count(tc.n0, r, w) + owned_count(tc.n1, r, w) + owned_count(tc.n2, r, w);
    const int ng = (P + kShardGran - 1) / kShardGran;
    const int cnt = owned_count(ng, r, w);
    m.np = cnt * kShardGran;
    if (cnt > 0 && (ng - 1) % w == r) m.np -= ng * kShardGran - P;  // this rank holds the partial last granule
    return m;
}
// Global packed token of local packed token i.
__host__ __device__ __forceinline__ int packed_global(int i, int r, int w) {
    return w <= 1 ? i : ((i / kShardGran) * w + r) * kShardGran + i % kShardGran;
}
// Tier (0 sinks, 1 heavy hitters, 2 ring) and slot of local dense position i.
__host__ __device__ __forceinline__ int dense_local_slot(const TierCounts& tc, int i, int r, int w, int& slot) {
    if (w <= 1) {
        if (i < tc.n0) { slot = i; return 0; }
        if (i < tc.n0 + tc.n1) { slot = i - tc.n0; return 1; }
        const int q = i - tc.n0 - tc.n1;
        slot = tc.ring_size > 0 ? (tc.ring_head + q) % tc.ring_size : q;  // logical ring order
        return 2;
    }
    const int a = owned_count(tc.n0, r, w), b = owned_count(tc.n1, r, w);
    if (i < a) { slot = r + w * i; return 0; }
    if (i < a + b) { slot = r + w * (i - a); return 1; }
    slot = r + w * (i - a - b);
    return 2;
}
// Ring slot -> token id: the ring holds ids [total - n2, total), the oldest
// at ring_head (ring_head is 0 while the ring fills).
__host__ __device__ __forceinline__ long long ring_slot_id(const TierCounts& tc, int slot) {
    int q = slot - tc.ring_head;
    if (q < 0) q += tc.ring_size;
    return (long long)tc.total - tc.n2 + q;
}

// Total order of floats as unsigned keys (negative values reversed), and back.
__host__ __device__ __forceinline__ uint32_t order_key(float x) {
    uint32_t b;
    memcpy(&b, &x, 4);
    return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}
__host__ __device__ __forceinline__ float key_value(uint32_t k) {
    const uint32_t b = (k & 0x80000000u) ? (k & 0x7fffffffu) : ~k;
    float x;
    memcpy(&x, &b, 4);
    return x;
}

// Routing row a rank publishes after a sharded step, for the next step's
// maintenance on every rank: the accumulated score of the token the next
// step evicts (valid from the owner of ring slot ring_head) and the smallest
// (score, slot) over this rank's heavy-hitter slots (slot -1: none).
struct RouteRow {
    float ev_score;
    float hh_min;
    int hh_slot;
    int pad;
};

// Flags across GPUs (system scope): a release store after the data it
// publishes, an acquire load before reading the data it guards.
__device__ __forceinline__ unsigned long long ld_acquire_sys(const unsigned long long* p) {
    unsigned long long v;
    asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void st_release_sys(unsigned long long* p, unsigned long long v) {
    asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
// Waits until f[q * stride] >= target for q < count; bounded (2^22 polls
// with a 256 ns sleep: a few seconds at most).  False if a wait ran out.
constexpr int kPeerSpin = 1 << 22;
__device__ __forceinline__ bool wait_peer_flags(const unsigned long long* f, int stride, int count, long long target) {
    for (int q = 0; q < count; ++q) {
        int it = 0;
        while ((long long)ld_acquire_sys(f + (size_t)q * stride) < target) {
            if (++it >= kPeerSpin) return false;
            __nanosleep(256);
        }
    }
    return true;
}

// Scratch a job needs for a given plan: chunk slots and score stride.
int attn_max_chunks(int dense_cap, int pbs_tok_cap);
// Launches the partial, head-merge and weights kernels on `stream`.
tt_status launch_attention(const AttnLaunch& L, cudaStream_t stream);

// Sequence-sharded attention, two stream-ordered phases around an all-gather
// done by the caller (L.rank / L.world set, L.mw unused):
//  1. partial attention over the tokens this rank owns, merged into one
//     (m, l, acc[hd]) row per (job, head): xch[job][h][hd + 2];
//  2. given every rank's rows (xch_all[world][njobs][nq][hd + 2]): the output
//     (same arithmetic and order on every rank), the score feedback of this
//     rank's tokens and its routing row route[job] for the next step.
tt_status launch_sharded_partial(const AttnLaunch& L, float* xch, cudaStream_t stream);
tt_status launch_sharded_merge(const AttnLaunch& L, const float* xch_all, RouteRow* route, int pos_cap,
                               cudaStream_t stream);

}  // namespace tt
