// tt_engine.cu -- device-resident TriTierCache engine.
//
// Replaces TriTierCacheEngine (csrc/cache_engine.cpp).  All tier buffers and
// counters live in HBM; one decode step is four stream-ordered launches for
// any number of engines (layers / sequences):
//   k_engine_maintain  one CTA per engine: ingest the new token into the
//                      sink / recent-window ring, evict the oldest ring slot,
//                      route it (radix-select percentile threshold every
//                      update_interval tokens, heavy-hitter append or
//                      strict-argmin replace with demotion), and flush a full
//                      waiting room into one packed block (bit-exact
//                      quantize+pack).  cache_engine.cpp:118-269, :397-431.
//   k_attn_dense + k_attn_packed (concurrent), then k_attn_weights
//                      (tt_attn.cu) over the tiers in place (no dense
//                      re-assembly, cache_engine.cpp:433-459), with the
//                      decayed score feedback fused into the weights pass
//                      (cache_engine.cpp:511-540).
// Sequence-sharded steps (tt_engine_step_sharded_*) run the same maintenance
// on every rank with routing inputs from the ranks' routing rows, the
// attention over the rank's own tokens, and k_shard_merge; the score
// synchronisation (k_scores_pack / k_scores_unpack) runs before the steps that
// recompute the heavy-hitter threshold.
// The host never waits for the device inside step(); the integer state the
// host needs for grid sizing is either deterministic (token counts) or an
// upper bound (packed blocks).
#include <algorithm>
#include <new>
#include <string.h>
#include <vector>

#include "tt_attn.cuh"

using namespace tt;

struct tt_engine {
    tt_engine_config cfg;
    int chunk, qhd, max_hh;
    size_t kvs;
    int meta_bytes;
    // device buffers
    float *S_K = nullptr, *S_V = nullptr, *RW_K = nullptr, *RW_V = nullptr, *HH_K = nullptr, *HH_V = nullptr;
    float *HH_scores = nullptr, *WR_K = nullptr, *WR_V = nullptr, *g = nullptr;
    int64_t *HH_ids = nullptr, *WR_ids = nullptr, *PBS_ids = nullptr;
    int32_t *kp = nullptr, *vp = nullptr;
    void *ks = nullptr, *kz = nullptr, *vs = nullptr, *vz = nullptr;
    int pbs_cap = 0;  // physical packed blocks
    DevCounters* ctr = nullptr;
    float* scratch = nullptr;
    size_t scratch_floats = 0;
    JobDesc* job_dev = nullptr;
    void* maint_dev = nullptr;
    int* full_map = nullptr;  // reconstruct: id -> tier slot, then the compacted id list
    size_t full_map_n = 0;
    // host mirrors: exact (token-count driven) and upper bounds
    int h_total = 0, h_s = 0, h_rw = 0, h_rw_head = 0, h_evictions = 0;
    int h_last_calc = -1;  // last_calc_pos: the steps that recompute the threshold
    long long h_wr_pbs_ub = 0;  // upper bound of tokens in waiting room + PBS
    cudaStream_t last_stream = nullptr;
};

// Peer-memory exchange of sequence-sharded steps: this rank's region (rows,
// routing rows, flags; see PeerXch) and the other ranks' regions opened
// through CUDA IPC.
struct tt_xch {
    int world = 0, rank = 0, jobs = 0, nq = 0, hd = 0, device = 0;
    size_t rows_bytes = 0, route_bytes = 0, flags_bytes = 0;
    char* base = nullptr;                       // own region
    char* peer[tt::kMaxWorld] = {nullptr};      // opened regions of the other ranks
    long long step = 0;
    bool opened = false;
};

namespace tt {

// Per-engine constants and pointers read by the maintenance kernel.
struct MaintDesc {
    int nkv, hd, msl, S, R, ui, grp, meta16, max_hh, qhd, pbs_cap;
    float h_ratio;
    size_t kvs;
    float *S_K, *S_V, *RW_K, *RW_V, *HH_K, *HH_V, *HH_scores, *WR_K, *WR_V, *g;
    int64_t *HH_ids, *WR_ids, *PBS_ids;
    int32_t *kp, *vp;
    void *ks, *kz, *vs, *vz;
    DevCounters* ctr;
};

struct MaintBatch {
    int n;
    // Sequence-sharded steps: the ranks' routing rows [world][n] of the last
    // step (nullptr: route from this engine's own scores, which are then
    // current for every token).
    const RouteRow* route;
    int world;
    int route_stride;                      // rows between ranks' slots of `route`
    const unsigned long long* route_flags; // peer exchange: wait for flags[q * route_stride + job] >= route_step
    long long route_step;
    const MaintDesc* d[kMaxBatch];
    const float* K[kMaxBatch];
    const float* V[kMaxBatch];
};

constexpr int MT = 512;  // maintenance CTA size

__device__ __forceinline__ void copy_row(float* __restrict__ dst, const float* __restrict__ src, size_t n) {
    if ((((uintptr_t)dst | (uintptr_t)src) & 15) == 0 && (n & 3) == 0) {
        float4* d4 = reinterpret_cast<float4*>(dst);
        const float4* s4 = reinterpret_cast<const float4*>(src);
        for (size_t i = threadIdx.x; i < n / 4; i += blockDim.x) d4[i] = s4[i];
    } else {
        for (size_t i = threadIdx.x; i < n; i += blockDim.x) dst[i] = src[i];
    }
}

// k-th smallest (0-based) of x[0..n): 4 passes of an 8-bit radix histogram.
// Returns the same value as std::nth_element (cache_engine.cpp:140-141).  The
// histograms are per warp (hist: [blockDim.x / 32][256] in shared memory), and
// the lanes of a warp whose keys fall in one bin add once (match_any), so
// equal scores -- most of them share their top bytes -- do not serialise on
// one shared-memory word; warp 0 then sums the warps' histograms, 8 bins per
// lane, and finds the bin holding k with one scan over the lanes.
constexpr int kSelU = 16;  // candidates per thread per round of the radix select
__device__ float block_select_kth(const float* __restrict__ x, int n, int k, unsigned int* hist) {
    __shared__ uint32_t s_prefix, s_k;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    unsigned int* hw = hist + warp * 256;
    uint32_t prefix = 0, mask = 0;
    if (threadIdx.x == 0) s_k = (uint32_t)k;
    for (int pass = 0; pass < 4; ++pass) {
        const int shift = 24 - 8 * pass;
        for (int i = threadIdx.x; i < nw * 256; i += blockDim.x) hist[i] = 0;
        __syncthreads();
        // whole warps step together, kSelU loads in flight per thread (one CTA
        // reads all the candidates four times: latency, not bandwidth, bounds it)
        for (int base = warp * 32 * kSelU; base < n; base += blockDim.x * kSelU) {
            float v[kSelU];
#pragma unroll
            for (int u = 0; u < kSelU; ++u) {
                const int i = base + 32 * u + lane;
                v[u] = i < n ? __ldcg(x + i) : 0.f;
            }
#pragma unroll
            for (int u = 0; u < kSelU; ++u) {
                uint32_t bin = 0xffffffffu;  // none
                if (base + 32 * u + lane < n) {
                    const uint32_t key = order_key(v[u]);
                    if ((key & mask) == prefix) bin = (key >> shift) & 255u;
                }
                const unsigned grp = __match_any_sync(0xffffffffu, bin);
                if (bin != 0xffffffffu && lane == __ffs(grp) - 1) atomicAdd(&hw[bin], (unsigned)__popc(grp));
            }
        }
        __syncthreads();
        if (warp == 0) {
            uint32_t c[8], tot = 0;
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                uint32_t t = 0;
                for (int w = 0; w < nw; ++w) t += hist[w * 256 + lane * 8 + j];
                c[j] = t;
                tot += t;
            }
            uint32_t incl = tot;  // inclusive scan of the lanes' totals
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const uint32_t v = __shfl_up_sync(0xffffffffu, incl, o);
                if (lane >= o) incl += v;
            }
            const uint32_t excl = incl - tot, kk = s_k;
            const bool mine = kk >= excl && kk < incl;
            const unsigned who = __ballot_sync(0xffffffffu, mine);
            if (mine) {
                uint32_t cum = excl;
                int d = 0;
                for (; d < 8; ++d) {
                    if (kk < cum + c[d]) break;
                    cum += c[d];
                }
                s_k = kk - cum;
                s_prefix = prefix | ((uint32_t)(lane * 8 + d) << shift);
            }
            const uint32_t all = __shfl_sync(0xffffffffu, incl, 31);
            if (who == 0 && lane == 0) {  // k at or past the count (not reached for k < n): the last bin
                s_k = kk - all;
                s_prefix = prefix | (255u << shift);
            }
        }
        __syncthreads();
        prefix = s_prefix;
        mask |= 255u << shift;
        __syncthreads();
    }
    return key_value(prefix);
}

// quantize the full waiting room into packed block `b` (cache_engine.cpp:148-207)
__device__ void flush_waiting_room(const MaintDesc& E, DevCounters& c) {
    const int b = c.pbs_used;
    if (b >= E.pbs_cap) {  // the host sizes the PBS from an upper bound; never expected
        if (threadIdx.x == 0) c.error = TT_ERR_OUT_OF_RANGE;
        __syncthreads();
        return;
    }
    if (threadIdx.x == 0 && b + 1 > c.pbs_alloc) c.pbs_alloc = max(c.pbs_alloc + 64, b + 1);  // :84-116
    const size_t words = (size_t)E.grp / 16;
    const size_t mbytes = E.meta16 ? 2 : 4;
    quantize_k_block_dev(E.WR_K, reinterpret_cast<uint32_t*>(E.kp) + (size_t)b * words * E.kvs,
                         (char*)E.ks + (size_t)b * E.kvs * mbytes, (char*)E.kz + (size_t)b * E.kvs * mbytes,
                         E.meta16, E.nkv, E.hd, E.grp, threadIdx.x, blockDim.x);
    const size_t vm = (size_t)b * E.grp * E.nkv;
    quantize_v_block_dev(E.WR_V, E.vp + vm * E.qhd, (char*)E.vs + vm * mbytes, (char*)E.vz + vm * mbytes, E.meta16,
                         E.nkv, E.hd, E.grp, threadIdx.x, blockDim.x);
    for (int t = threadIdx.x; t < E.grp; t += blockDim.x) E.PBS_ids[(size_t)b * E.grp + t] = E.WR_ids[t];
    __syncthreads();
    if (threadIdx.x == 0) {
        c.pbs_used = b + 1;
        c.pbs_count += E.grp;
        c.wr_count = 0;
    }
    __syncthreads();
}

__global__ void __launch_bounds__(MT) k_engine_maintain(const __grid_constant__ MaintBatch B) {
    __shared__ MaintDesc E;
    __shared__ DevCounters c;
    __shared__ unsigned int hist[(MT / 32) * 256];  // per-warp radix histograms
    __shared__ float s_red_v[MT / 32];
    __shared__ int s_red_i[MT / 32];
    __shared__ int s_action, s_mi;
    __shared__ float s_score;
    if (threadIdx.x == 0) {
        E = *B.d[blockIdx.x];
        // peer exchange: every rank's routing row of the last step has landed
        if (B.route && B.route_flags &&
            !wait_peer_flags(B.route_flags + blockIdx.x, B.route_stride, B.world, B.route_step)) {
            atomicCAS(&E.ctr->error, 0, (int)TT_ERR_TIMEOUT);  // the engine's sticky error
        }
        c = *E.ctr;
    }
    __syncthreads();
    const float* Kn = B.K[blockIdx.x];
    const float* Vn = B.V[blockIdx.x];
    const size_t kvs = E.kvs;

    if (c.s_count < E.S) {  // :406-409
        copy_row(E.S_K + (size_t)c.s_count * kvs, Kn, kvs);
        copy_row(E.S_V + (size_t)c.s_count * kvs, Vn, kvs);
        __syncthreads();
        if (threadIdx.x == 0) c.s_count++;
    } else if (c.rw_count < E.R) {  // :410-413
        copy_row(E.RW_K + (size_t)c.rw_count * kvs, Kn, kvs);
        copy_row(E.RW_V + (size_t)c.rw_count * kvs, Vn, kvs);
        __syncthreads();
        if (threadIdx.x == 0) c.rw_count++;
    } else {
        // ---- ring eviction (:414-430) and routing (:209-269) ----
        const int slot = c.rw_head;
        const long long id = (long long)c.total - E.R;
        const float* ek = E.RW_K + (size_t)slot * kvs;
        const float* ev = E.RW_V + (size_t)slot * kvs;
        // threshold (:118-146); candidates clamped to the score buffer
        const int cs = E.S, ce = c.total - E.R;
        if (ce <= cs) {
            if (threadIdx.x == 0) c.cached_threshold = 0.f;
        } else if (c.last_calc_pos == -1 || (c.total - c.last_calc_pos >= E.ui)) {
            const int n = ce - cs;
            float q = 1.0f - E.h_ratio;
            q = q < 0.f ? 0.f : (q > 1.f ? 1.f : q);
            const int k = (int)(size_t)(q * (float)(n - 1));
            const int nread = min(ce, E.msl) - cs;
            const float v = nread > 0 ? block_select_kth(E.g + cs, nread, min(k, nread - 1), hist) : 0.f;
            if (threadIdx.x == 0) {
                c.cached_threshold = v;
                c.last_calc_pos = c.total;
            }
        }
        __syncthreads();
        if (threadIdx.x == 0) {
            c.total_evictions++;
            if (B.route) {
                // the ring slot's owner published the score; every rank stores
                // it, so the token's score is current wherever it moves next
                s_score = B.route[(size_t)(slot % B.world) * B.route_stride + blockIdx.x].ev_score;
                if (id >= 0 && id < E.msl) E.g[id] = s_score;
            } else {
                s_score = (id >= 0 && id < E.msl) ? E.g[id] : 0.f;
            }
        }
        __syncthreads();
        const float score = s_score, thresh = c.cached_threshold;
        int action = 2;  // 0: HH append, 1: HH replace + demote, 2: waiting room
        int mi = 0;
        if (score >= thresh) {
            if (c.hh_count < E.max_hh) {
                action = 0;
            } else if (B.route) {
                // global strict-< argmin, first slot wins: the smallest
                // (score, slot) over the ranks' minima of their own slots
                if (threadIdx.x == 0) {
                    float v0 = INFINITY;
                    int i0 = -1;
                    for (int p = 0; p < B.world; ++p) {
                        const RouteRow rr = B.route[(size_t)p * B.route_stride + blockIdx.x];
                        if (rr.hh_slot >= 0 && (i0 < 0 || rr.hh_min < v0 || (rr.hh_min == v0 && rr.hh_slot < i0))) {
                            v0 = rr.hh_min;
                            i0 = rr.hh_slot;
                        }
                    }
                    s_mi = i0 < 0 ? 0 : i0;
                    s_action = (i0 >= 0 && score > v0) ? 1 : 2;
                    if (s_action == 1) {  // the demoted token's current score (its owner's HH_scores entry)
                        const long long did = E.HH_ids[i0];
                        if (did >= 0 && did < E.msl) E.g[did] = v0;
                    }
                }
                __syncthreads();
                action = s_action;
                mi = s_mi;
            } else {
                // strict-< argmin, first index wins (:231-238)
                float bv = INFINITY;
                int bi = 0x7fffffff;  // "none"
                for (int i = threadIdx.x; i < c.hh_count; i += blockDim.x) {
                    const float v = E.HH_scores[i];
                    if (bi == 0x7fffffff || v < bv) { bv = v; bi = i; }  // i ascends: ties keep the first
                }
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) {
                    const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
                    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
                    if (oi != 0x7fffffff && (bi == 0x7fffffff || ov < bv || (ov == bv && oi < bi))) { bv = ov; bi = oi; }
                }
                if ((threadIdx.x & 31) == 0) { s_red_v[threadIdx.x >> 5] = bv; s_red_i[threadIdx.x >> 5] = bi; }
                __syncthreads();
                if (threadIdx.x == 0) {
                    float v0 = INFINITY;
                    int i0 = 0x7fffffff;
                    for (int w = 0; w < (int)(blockDim.x >> 5); ++w) {
                        const int oi = s_red_i[w];
                        const float ov = s_red_v[w];
                        if (oi != 0x7fffffff && (i0 == 0x7fffffff || ov < v0 || (ov == v0 && oi < i0))) { v0 = ov; i0 = oi; }
                    }
                    s_mi = i0;
                    s_action = (score > v0) ? 1 : 2;
                }
                __syncthreads();
                action = s_action;
                mi = s_mi;
            }
        }
        if (action == 0) {
            const int h = c.hh_count;
            copy_row(E.HH_K + (size_t)h * kvs, ek, kvs);
            copy_row(E.HH_V + (size_t)h * kvs, ev, kvs);
            if (threadIdx.x == 0) {
                E.HH_ids[h] = id;
                E.HH_scores[h] = score;
            }
            __syncthreads();
            if (threadIdx.x == 0) c.hh_count = h + 1;
        } else if (action == 1) {
            const int w = c.wr_count;
            copy_row(E.WR_K + (size_t)w * kvs, E.HH_K + (size_t)mi * kvs, kvs);
            copy_row(E.WR_V + (size_t)w * kvs, E.HH_V + (size_t)mi * kvs, kvs);
            if (threadIdx.x == 0) E.WR_ids[w] = E.HH_ids[mi];
            __syncthreads();
            copy_row(E.HH_K + (size_t)mi * kvs, ek, kvs);
            copy_row(E.HH_V + (size_t)mi * kvs, ev, kvs);
            if (threadIdx.x == 0) {
                E.HH_ids[mi] = id;
                E.HH_scores[mi] = score;
                c.wr_count = w + 1;
            }
            __syncthreads();
        } else {
            const int w = c.wr_count;
            copy_row(E.WR_K + (size_t)w * kvs, ek, kvs);
            copy_row(E.WR_V + (size_t)w * kvs, ev, kvs);
            if (threadIdx.x == 0) {
                E.WR_ids[w] = id;
                c.wr_count = w + 1;
            }
            __syncthreads();
        }
        __syncthreads();
        if (c.wr_count == E.grp) flush_waiting_room(E, c);
        // overwrite the ring slot with the new token (:424-428)
        copy_row(E.RW_K + (size_t)slot * kvs, Kn, kvs);
        copy_row(E.RW_V + (size_t)slot * kvs, Vn, kvs);
        __syncthreads();
        if (threadIdx.x == 0) c.rw_head = (c.rw_head + 1) % E.R;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        c.total++;
        *E.ctr = c;
    }
}

// ---------------------------------------------------------------------------
// prefill (cache_engine.cpp:271-395)
// ---------------------------------------------------------------------------
// grid = blocks to quantize; block b reads tokens [S + b*C, +C) into packed
// block (pbs_used + b).
__global__ void __launch_bounds__(256) k_prefill_quantize(const MaintDesc* __restrict__ Ed, const float* K_all,
                                                         const float* V_all) {
    const MaintDesc& E = *Ed;
    const int base = E.ctr->pbs_used;
    const int b = blockIdx.x;
    const int dst = base + b;
    if (dst >= E.pbs_cap) return;
    const int src = E.S + b * E.grp;
    const size_t words = (size_t)E.grp / 16;
    const size_t mbytes = E.meta16 ? 2 : 4;
    quantize_k_block_dev(K_all + (size_t)src * E.kvs, reinterpret_cast<uint32_t*>(E.kp) + (size_t)dst * words * E.kvs,
                         (char*)E.ks + (size_t)dst * E.kvs * mbytes, (char*)E.kz + (size_t)dst * E.kvs * mbytes,
                         E.meta16, E.nkv, E.hd, E.grp, threadIdx.x, blockDim.x);
    const size_t vm = (size_t)dst * E.grp * E.nkv;
    quantize_v_block_dev(V_all + (size_t)src * E.kvs, E.vp + vm * E.qhd, (char*)E.vs + vm * mbytes,
                         (char*)E.vz + vm * mbytes, E.meta16, E.nkv, E.hd, E.grp, threadIdx.x, blockDim.x);
    for (int t = threadIdx.x; t < E.grp; t += blockDim.x) E.PBS_ids[(size_t)dst * E.grp + t] = src + t;
}

// tier copies and counter updates; runs after k_prefill_quantize
__global__ void __launch_bounds__(512) k_prefill_finish(const MaintDesc* __restrict__ Ed, const float* K_all,
                                                       const float* V_all, int q_len, int nblk) {
    const MaintDesc& E = *Ed;
    __shared__ DevCounters c;
    if (threadIdx.x == 0) c = *E.ctr;
    __syncthreads();
    const size_t kvs = E.kvs;
    if (q_len <= E.S + E.R) {
        const int s = min(E.S, q_len);
        if (s > 0) {
            copy_row(E.S_K, K_all, (size_t)s * kvs);
            copy_row(E.S_V, V_all, (size_t)s * kvs);
        }
        const int r = q_len - s;
        if (r > 0) {
            copy_row(E.RW_K, K_all + (size_t)s * kvs, (size_t)r * kvs);
            copy_row(E.RW_V, V_all + (size_t)s * kvs, (size_t)r * kvs);
        }
        __syncthreads();
        if (threadIdx.x == 0) {
            if (s > 0) c.s_count = s;
            if (r > 0) { c.rw_count = r; c.rw_head = 0; }
            c.total = q_len;
            *E.ctr = c;
        }
        return;
    }
    copy_row(E.S_K, K_all, (size_t)E.S * kvs);
    copy_row(E.S_V, V_all, (size_t)E.S * kvs);
    const int rw_start = q_len - E.R;
    copy_row(E.RW_K, K_all + (size_t)rw_start * kvs, (size_t)E.R * kvs);
    copy_row(E.RW_V, V_all + (size_t)rw_start * kvs, (size_t)E.R * kvs);
    const int n_inter = rw_start - E.S;
    const int rem = n_inter - nblk * E.grp;
    if (rem > 0) {
        const int rs = E.S + nblk * E.grp;
        copy_row(E.WR_K, K_all + (size_t)rs * kvs, (size_t)rem * kvs);
        copy_row(E.WR_V, V_all + (size_t)rs * kvs, (size_t)rem * kvs);
        for (int t = threadIdx.x; t < rem; t += blockDim.x) E.WR_ids[t] = rs + t;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        c.s_count = E.S;
        c.rw_count = E.R;
        c.rw_head = 0;
        if (nblk > 0) {
            const int need = c.pbs_used + nblk;
            if (need > E.pbs_cap) c.error = TT_ERR_OUT_OF_RANGE;
            if (need > c.pbs_alloc) c.pbs_alloc = max(c.pbs_alloc + 64, need);
            c.pbs_used = need;
            c.pbs_count += nblk * E.grp;
            c.total_evictions += nblk * E.grp;
        }
        c.wr_count = rem > 0 ? rem : 0;
        c.total = q_len;
        *E.ctr = c;
    }
}

__global__ void k_fill_i64(int64_t* p, size_t n, int64_t v) {
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) p[i] = v;
}

}  // namespace tt

// ---------------------------------------------------------------------------
// full-cache reconstruction and undecayed score accumulation (the reference's
// output_attentions path, src/tri_tier/cache.py:164-187 and :326-372)
// ---------------------------------------------------------------------------
// map[id - lo] = tier slot of every middle token: heavy-hitter slot i -> i,
// live packed position p -> max_hh + p (ids are unique across tiers).
__global__ void k_full_map(const int64_t* __restrict__ hh_ids, int hh, const int64_t* __restrict__ pbs_ids,
                           int npbs, int max_hh, long long lo, int n, int* __restrict__ map) {
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < hh + npbs; i += gridDim.x * blockDim.x) {
        const long long id = i < hh ? hh_ids[i] : pbs_ids[i - hh];
        const long long j = id - lo;
        if (id >= 0 && j >= 0 && j < n) map[j] = i < hh ? i : max_hh + (i - hh);
    }
}

// One CTA: compacts the present entries of map[0..n) in id order into
// list[0..count) (their map indices) and writes count.  1024 threads, each a
// contiguous run, one block-wide scan of the run counts.
__global__ void __launch_bounds__(1024) k_full_compact(const int* __restrict__ map, int n, int* __restrict__ list,
                                                       int* __restrict__ count) {
    __shared__ int warp_tot[32];
    const int per = (n + blockDim.x - 1) / blockDim.x;
    const int a = min(n, (int)threadIdx.x * per), b = min(n, a + per);
    int c = 0;
    for (int j = a; j < b; ++j) c += map[j] >= 0;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    int x = c;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, x, o);
        if (lane >= o) x += y;
    }
    if (lane == 31) warp_tot[warp] = x;
    __syncthreads();
    if (warp == 0) {
        int t = lane < (int)(blockDim.x >> 5) ? warp_tot[lane] : 0;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int y = __shfl_up_sync(0xffffffffu, t, o);
            if (lane >= o) t += y;
        }
        warp_tot[lane] = t;  // inclusive prefix over warps
    }
    __syncthreads();
    int pos = x - c + (warp > 0 ? warp_tot[warp - 1] : 0);  // exclusive prefix of this thread's run
    for (int j = a; j < b; ++j)
        if (map[j] >= 0) list[pos++] = j;
    if (threadIdx.x == blockDim.x - 1) *count = pos;
}

// Rows [sinks | middle tokens by id | ring in logical order] of the full cache,
// packed tokens dequantized as code * scale + zero with two roundings (the
// reference's torch expression, cache.py:336-345).
__global__ void k_full_gather(const MaintDesc* __restrict__ Ed, int S, int nmid, int rw, int head, long long total,
                              long long lo, const int* __restrict__ map, const int* __restrict__ list,
                              float* __restrict__ Ko, float* __restrict__ Vo, int64_t* __restrict__ ids) {
    const MaintDesc& E = *Ed;
    const int rows = S + nmid + rw;
    const size_t kvs = E.kvs;
    const int hd = E.hd;
    for (size_t x = (size_t)blockIdx.x * blockDim.x + threadIdx.x; x < (size_t)rows * kvs;
         x += (size_t)gridDim.x * blockDim.x) {
        const int r = (int)(x / kvs);
        const size_t e = x % kvs;
        float kv, vv;
        long long id;
        if (r < S) {
            kv = E.S_K[(size_t)r * kvs + e];
            vv = E.S_V[(size_t)r * kvs + e];
            id = r;
        } else if (r < S + nmid) {
            const int j = list[r - S];
            const int slot = map[j];
            id = lo + j;
            if (slot < E.max_hh) {
                kv = E.HH_K[(size_t)slot * kvs + e];
                vv = E.HH_V[(size_t)slot * kvs + e];
            } else {
                const int p = slot - E.max_hh;             // packed token position
                const int b = p / E.grp, t = p % E.grp;    // block, token within the block
                const int h = (int)(e / hd), c = (int)(e % hd);
                const uint32_t kw = reinterpret_cast<const uint32_t*>(E.kp)[((size_t)b * (E.grp / 16) + t / 16) * kvs + e];
                const float ks = load_meta(E.ks, (size_t)b * kvs + e, E.meta16);
                const float kz = load_meta(E.kz, (size_t)b * kvs + e, E.meta16);
                kv = __fadd_rn(__fmul_rn((float)((kw >> (2 * (t % 16))) & 3u), ks), kz);
                const uint32_t vw = reinterpret_cast<const uint32_t*>(E.vp)[((size_t)p * E.nkv + h) * E.qhd + c / 16];
                const float vs = load_meta(E.vs, (size_t)p * E.nkv + h, E.meta16);
                const float vz = load_meta(E.vz, (size_t)p * E.nkv + h, E.meta16);
                vv = __fadd_rn(__fmul_rn((float)((vw >> (2 * (c % 16))) & 3u), vs), vz);
            }
        } else {
            const int i = r - S - nmid;
            const int slot = rw == E.R ? (head + i) % E.R : i;
            kv = E.RW_K[(size_t)slot * kvs + e];
            vv = E.RW_V[(size_t)slot * kvs + e];
            id = rw == E.R ? total - E.R + i : (long long)S + i;
        }
        Ko[x] = kv;
        Vo[x] = vv;
        if (e == 0) ids[r] = id;
    }
}

// g[ids[i]] += (1/H) sum_h w[h][i] for ids[i] in [0, msl) (cache.py:164-187:
// mean over heads, index_add_ without decay).  Ids are unique, so no two
// threads add to one entry.
__global__ void k_accumulate_scores(float* __restrict__ g, int msl, const float* __restrict__ w,
                                    const int64_t* __restrict__ ids, int H, int n) {
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
        const long long id = ids ? ids[i] : i;
        if (id < 0 || id >= msl) continue;
        float s = 0.f;
        for (int h = 0; h < H; ++h) s += w[(size_t)h * n + i];
        g[id] += s / (float)H;
    }
}

// ---------------------------------------------------------------------------
// score synchronisation of sequence-sharded steps
// ---------------------------------------------------------------------------
// Engines of one synchronisation and the offset of each one's scores in the
// exchanged buffer ([sum of max_seq_len] floats, engine after engine).
struct ScoreBatch {
    int n;
    const MaintDesc* d[kMaxBatch];
    long long off[kMaxBatch];
};

// buf[id] = g[id] for the tokens rank `r` of `w` owns (zero elsewhere; the
// caller zeroes buf): its sink, heavy-hitter and ring slots (slot % w == r),
// its packed granules, and on rank 0 the waiting room, whose scores every
// rank holds.  Summed over the ranks, buf is every token's current score.
// grid (gx, engines).
__global__ void __launch_bounds__(256) k_scores_pack(const __grid_constant__ ScoreBatch B, int r, int w,
                                                     float* __restrict__ buf_all) {
    const MaintDesc& E = *B.d[blockIdx.y];
    float* buf = buf_all + B.off[blockIdx.y];
    const DevCounters c = *E.ctr;
    TierCounts tc;
    tc.n0 = c.s_count; tc.n1 = c.hh_count; tc.n2 = c.rw_count; tc.ring_head = c.rw_head; tc.ring_size = E.R;
    tc.nblk = c.pbs_used; tc.total = c.total;
    const long long nS = E.S, nH = E.max_hh, nR = E.R, nW = E.grp;
    const long long nP = (long long)c.pbs_used * E.grp;
    const long long items = nS + nH + nR + nW + nP;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < items;
         i += (long long)gridDim.x * blockDim.x) {
        long long id = -1;
        if (i < nS) {
            if (i < tc.n0 && i % w == r) id = i;
        } else if (i < nS + nH) {
            const int k = (int)(i - nS);
            if (k < tc.n1 && k % w == r) id = E.HH_ids[k];
        } else if (i < nS + nH + nR) {
            const int k = (int)(i - nS - nH);
            if (k < tc.n2 && k % w == r) id = ring_slot_id(tc, k);
        } else if (i < nS + nH + nR + nW) {
            const int k = (int)(i - nS - nH - nR);
            if (k < c.wr_count && r == 0) id = E.WR_ids[k];
        } else {
            const long long p = i - nS - nH - nR - nW;
            if ((p / kShardGran) % w == r) id = E.PBS_ids[p];
        }
        if (id >= 0 && id < E.msl) buf[id] = E.g[id];
    }
}

// g = buf and HH_scores[i] = buf[HH_ids[i]] (the heavy hitters' copy of the
// synchronised scores).  grid (gx, engines).
__global__ void __launch_bounds__(256) k_scores_unpack(const __grid_constant__ ScoreBatch B,
                                                       const float* __restrict__ buf_all) {
    const MaintDesc& E = *B.d[blockIdx.y];
    const float* buf = buf_all + B.off[blockIdx.y];
    const int nh = E.ctr->hh_count;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < E.msl;
         i += (long long)gridDim.x * blockDim.x)
        E.g[i] = buf[i];
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < nh; i += gridDim.x * blockDim.x) {
        const long long id = E.HH_ids[i];
        if (id >= 0 && id < E.msl) E.HH_scores[i] = buf[id];
    }
}

// ---------------------------------------------------------------------------
// host
// ---------------------------------------------------------------------------
namespace {

struct DeviceGuard {
    int prev = -1;
    explicit DeviceGuard(int dev) {
        cudaGetDevice(&prev);
        if (prev != dev) cudaSetDevice(dev);
    }
    ~DeviceGuard() {
        int cur = -1;
        cudaGetDevice(&cur);
        if (prev >= 0 && cur != prev) cudaSetDevice(prev);
    }
};

template <typename T>
tt_status dalloc(T** p, size_t n, const char* what) {
    *p = nullptr;
    if (n == 0) n = 1;
    tt_status s = check_cuda(cudaMalloc((void**)p, n * sizeof(T)), what);
    if (s != TT_OK) return s;
    return check_cuda(cudaMemset(*p, 0, n * sizeof(T)), what);
}

constexpr int kLogicalSlack = 64;

int dense_cap(const tt_engine* e) { return e->cfg.sink_size + e->max_hh + e->cfg.rw_size; }

void free_pbs(tt_engine* e) {
    cudaFree(e->kp); cudaFree(e->vp); cudaFree(e->ks); cudaFree(e->kz); cudaFree(e->vs); cudaFree(e->vz);
    cudaFree(e->PBS_ids);
    e->kp = e->vp = nullptr;
    e->ks = e->kz = e->vs = e->vz = nullptr;
    e->PBS_ids = nullptr;
}

tt_status write_descriptors(tt_engine* e) {
    MaintDesc md;
    md.nkv = e->cfg.num_kv_heads; md.hd = e->cfg.head_dim; md.msl = e->cfg.max_seq_len; md.S = e->cfg.sink_size;
    md.R = e->cfg.rw_size; md.ui = e->cfg.update_interval; md.grp = e->chunk; md.meta16 = e->cfg.meta_fp16;
    md.max_hh = e->max_hh; md.qhd = e->qhd; md.pbs_cap = e->pbs_cap; md.h_ratio = e->cfg.h_ratio; md.kvs = e->kvs;
    md.S_K = e->S_K; md.S_V = e->S_V; md.RW_K = e->RW_K; md.RW_V = e->RW_V; md.HH_K = e->HH_K; md.HH_V = e->HH_V;
    md.HH_scores = e->HH_scores; md.WR_K = e->WR_K; md.WR_V = e->WR_V; md.g = e->g;
    md.HH_ids = e->HH_ids; md.WR_ids = e->WR_ids; md.PBS_ids = e->PBS_ids;
    md.kp = e->kp; md.vp = e->vp; md.ks = e->ks; md.kz = e->kz; md.vs = e->vs; md.vz = e->vz; md.ctr = e->ctr;

    JobDesc j;
    memset(&j, 0, sizeof(j));
    j.nq = e->cfg.num_q_heads; j.nkv = e->cfg.num_kv_heads; j.hd = e->cfg.head_dim; j.grp = e->chunk;
    j.meta16 = e->cfg.meta_fp16; j.ring_size = e->cfg.rw_size;
    j.K0 = e->S_K; j.V0 = e->S_V; j.K1 = e->HH_K; j.V1 = e->HH_V; j.K2 = e->RW_K; j.V2 = e->RW_V;
    j.kp = e->kp; j.ks = e->ks; j.kz = e->kz; j.vp = e->vp; j.vs = e->vs; j.vz = e->vz; j.ids = e->PBS_ids;
    j.ctr = e->ctr;
    const int maxch = attn_max_chunks(dense_cap(e), e->pbs_cap * e->chunk);
    j.max_chunks = maxch;
    j.score_stride = (dense_cap(e) + e->pbs_cap * e->chunk + 3) / 4 * 4;  // float4 logit rows
    j.part_ml = e->scratch;
    j.part_acc = e->scratch + ((size_t)maxch * j.nq * 2 + 3) / 4 * 4;  // 16-byte aligned (float4 reads)
    j.scores = j.part_acc + (size_t)maxch * j.nq * j.hd;
    j.g = e->g; j.hh_scores = e->HH_scores; j.hh_ids = e->HH_ids; j.decay = e->cfg.score_decay;
    j.msl = e->cfg.max_seq_len;
    tt_status s = check_cuda(cudaMemcpy(e->maint_dev, &md, sizeof(md), cudaMemcpyHostToDevice), "descriptor upload");
    if (s != TT_OK) return s;
    return check_cuda(cudaMemcpy(e->job_dev, &j, sizeof(j), cudaMemcpyHostToDevice), "descriptor upload");
}

size_t scratch_need(const tt_engine* e, int pbs_cap) {
    const int maxch = attn_max_chunks(dense_cap(e), pbs_cap * e->chunk);
    const size_t stride = ((size_t)dense_cap(e) + (size_t)pbs_cap * e->chunk + 3) / 4 * 4;
    return (size_t)maxch * e->cfg.num_q_heads * (e->cfg.head_dim + 2) + (size_t)e->cfg.num_q_heads * stride + 64;
}

// (Re)allocates packed storage for `blocks` physical blocks, preserving
// the first `keep` blocks.  Synchronises the device (rare: the initial
// capacity covers max_seq_len tokens).
tt_status grow_pbs(tt_engine* e, int blocks) {
    const int old = e->pbs_cap;
    const size_t kvs = e->kvs, C = e->chunk, words = C / 16, mb = e->meta_bytes;
    const size_t vrow = (size_t)e->cfg.num_kv_heads * e->qhd;
    int32_t *kp, *vp;
    void *ks, *kz, *vs, *vz;
    int64_t* ids;
    tt_status s;
    if ((s = check_cuda(cudaDeviceSynchronize(), "PBS growth")) != TT_OK) return s;
    if ((s = dalloc(&kp, (size_t)blocks * words * kvs, "PBS_K_Packed")) != TT_OK) return s;
    if ((s = dalloc((char**)&ks, (size_t)blocks * kvs * mb, "PBS_K_Scales")) != TT_OK) return s;
    if ((s = dalloc((char**)&kz, (size_t)blocks * kvs * mb, "PBS_K_Zeroes")) != TT_OK) return s;
    if ((s = dalloc(&vp, (size_t)blocks * C * vrow, "PBS_V_Packed")) != TT_OK) return s;
    if ((s = dalloc((char**)&vs, (size_t)blocks * C * e->cfg.num_kv_heads * mb, "PBS_V_Scales")) != TT_OK) return s;
    if ((s = dalloc((char**)&vz, (size_t)blocks * C * e->cfg.num_kv_heads * mb, "PBS_V_Zeroes")) != TT_OK) return s;
    if ((s = dalloc(&ids, (size_t)blocks * C, "PBS_token_ids")) != TT_OK) return s;
    k_fill_i64<<<64, 256>>>(ids, (size_t)blocks * C, -1);
    if (old > 0) {
        cudaMemcpy(kp, e->kp, (size_t)old * words * kvs * 4, cudaMemcpyDeviceToDevice);
        cudaMemcpy(ks, e->ks, (size_t)old * kvs * mb, cudaMemcpyDeviceToDevice);
        cudaMemcpy(kz, e->kz, (size_t)old * kvs * mb, cudaMemcpyDeviceToDevice);
        cudaMemcpy(vp, e->vp, (size_t)old * C * vrow * 4, cudaMemcpyDeviceToDevice);
        cudaMemcpy(vs, e->vs, (size_t)old * C * e->cfg.num_kv_heads * mb, cudaMemcpyDeviceToDevice);
        cudaMemcpy(vz, e->vz, (size_t)old * C * e->cfg.num_kv_heads * mb, cudaMemcpyDeviceToDevice);
        cudaMemcpy(ids, e->PBS_ids, (size_t)old * C * 8, cudaMemcpyDeviceToDevice);
    }
    free_pbs(e);
    e->kp = kp; e->ks = ks; e->kz = kz; e->vp = vp; e->vs = vs; e->vz = vz; e->PBS_ids = ids;
    e->pbs_cap = blocks;
    const size_t need = scratch_need(e, blocks);
    if (need > e->scratch_floats) {
        cudaFree(e->scratch);
        e->scratch = nullptr;
        if ((s = dalloc(&e->scratch, need, "attention scratch")) != TT_OK) return s;
        e->scratch_floats = need;
    }
    if ((s = check_launch("PBS id init")) != TT_OK) return s;
    // the chunk-slot layout follows the capacity: start from a zeroed scratch
    // (the attention kernel's per-job arrival counter must read 0)
    if ((s = check_cuda(cudaMemset(e->scratch, 0, e->scratch_floats * sizeof(float)), "scratch clear")) != TT_OK)
        return s;
    if ((s = write_descriptors(e)) != TT_OK) return s;
    return check_cuda(cudaDeviceSynchronize(), "PBS growth");
}

// Makes sure a step (extra_tokens = 1) or a prefill cannot run out of packed blocks.
tt_status ensure_capacity(tt_engine* e, long long wr_pbs_tokens_after) {
    // the reference grows its logical allocation by +64 blocks (cache_engine.cpp:84-116), so the
    // logical view (pbs_allocated_blocks) can run up to 63 blocks past the blocks in use
    const long long blocks = wr_pbs_tokens_after / e->chunk + 1 + kLogicalSlack;
    if (blocks <= e->pbs_cap) return TT_OK;
    long long nb = std::max<long long>(blocks, (long long)e->pbs_cap + e->pbs_cap / 4 + 64);
    if (nb > (1LL << 30) / std::max<size_t>(1, e->kvs)) return set_error(TT_ERR_OUT_OF_MEMORY, "PBS capacity overflow");
    return grow_pbs(e, (int)nb);
}

tt_status validate(const tt_engine* e) {
    if (!e) return set_error(TT_ERR_INVALID_ARGUMENT, "engine handle is NULL.");
    return TT_OK;
}

}  // namespace

extern "C" {

tt_status tt_engine_create(const tt_engine_config* cfg, tt_engine** out) {
    if (!cfg || !out) return set_error(TT_ERR_INVALID_ARGUMENT, "NULL argument.");
    *out = nullptr;
    const tt_engine_config& c = *cfg;
    if (c.num_q_heads <= 0 || c.num_kv_heads <= 0 || c.head_dim <= 0 || c.max_seq_len <= 0)
        return set_error(TT_ERR_INVALID_ARGUMENT, "num_q_heads, num_kv_heads, head_dim and max_seq_len must be positive.");
    if (c.sink_size < 0 || c.rw_size <= 0)
        return set_error(TT_ERR_INVALID_ARGUMENT, "sink_size must be >= 0 and rw_size > 0.");
    if (c.update_interval < 0) return set_error(TT_ERR_INVALID_ARGUMENT, "update_interval must be >= 0.");
    if (c.head_dim % 16 != 0)
        return set_error(TT_ERR_UNSUPPORTED, "head_dim must be a multiple of 16 (packed V rows).");
    AttnLaunch probe;
    memset(&probe, 0, sizeof(probe));
    probe.njobs = 1;
    tt_status s = plan_attention(probe, c.num_q_heads, c.num_kv_heads, c.head_dim, 1, 1);
    if (s != TT_OK) return s;

    DeviceGuard dg(c.device);
    tt_engine* e = new (std::nothrow) tt_engine();
    if (!e) return set_error(TT_ERR_OUT_OF_MEMORY, "engine allocation failed");
    e->cfg = c;
    e->cfg.k_group_size = (c.k_group_size == 32) ? 32 : 16;  // cache_engine.cpp:29
    e->cfg.meta_fp16 = c.meta_fp16 ? 1 : 0;
    e->chunk = e->cfg.k_group_size;
    e->qhd = (c.head_dim + 15) / 16;
    e->max_hh = (int)ceilf((float)c.max_seq_len * c.h_ratio);  // :47-48
    if (e->max_hh < 1) e->max_hh = 1;
    e->kvs = (size_t)c.num_kv_heads * c.head_dim;
    e->meta_bytes = e->cfg.meta_fp16 ? 2 : 4;
    const size_t kvs = e->kvs;
#define TT_TRY(x)                     \
    do {                              \
        tt_status _s = (x);           \
        if (_s != TT_OK) {            \
            tt_engine_destroy(e);     \
            return _s;                \
        }                             \
    } while (0)
    TT_TRY(dalloc(&e->S_K, (size_t)std::max(c.sink_size, 1) * kvs, "S_K"));
    TT_TRY(dalloc(&e->S_V, (size_t)std::max(c.sink_size, 1) * kvs, "S_V"));
    TT_TRY(dalloc(&e->RW_K, (size_t)c.rw_size * kvs, "RW_K"));
    TT_TRY(dalloc(&e->RW_V, (size_t)c.rw_size * kvs, "RW_V"));
    TT_TRY(dalloc(&e->HH_K, (size_t)e->max_hh * kvs, "HH_K"));
    TT_TRY(dalloc(&e->HH_V, (size_t)e->max_hh * kvs, "HH_V"));
    TT_TRY(dalloc(&e->HH_scores, (size_t)e->max_hh, "HH_scores"));
    TT_TRY(dalloc(&e->HH_ids, (size_t)e->max_hh, "HH_token_ids"));
    TT_TRY(dalloc(&e->WR_K, (size_t)e->chunk * kvs, "WR_K"));
    TT_TRY(dalloc(&e->WR_V, (size_t)e->chunk * kvs, "WR_V"));
    TT_TRY(dalloc(&e->WR_ids, (size_t)e->chunk, "WR_token_ids"));
    TT_TRY(dalloc(&e->g, (size_t)c.max_seq_len, "global_attn_scores"));
    TT_TRY(dalloc(&e->ctr, 1, "counters"));
    TT_TRY(dalloc((char**)&e->maint_dev, sizeof(MaintDesc), "descriptor"));
    TT_TRY(dalloc((char**)&e->job_dev, sizeof(JobDesc), "descriptor"));
    k_fill_i64<<<8, 256>>>(e->HH_ids, (size_t)e->max_hh, -1);
    k_fill_i64<<<1, 64>>>(e->WR_ids, (size_t)e->chunk, -1);
    TT_TRY(check_launch("engine init"));
    DevCounters dc;
    memset(&dc, 0, sizeof(dc));
    dc.last_calc_pos = -1;
    TT_TRY(check_cuda(cudaMemcpy(e->ctr, &dc, sizeof(dc), cudaMemcpyHostToDevice), "counter init"));
    // packed capacity for max_seq_len tokens up front; grows only beyond that
    TT_TRY(grow_pbs(e, c.max_seq_len / e->chunk + 2 + kLogicalSlack));
    TT_TRY(check_cuda(cudaDeviceSynchronize(), "engine create"));
#undef TT_TRY
    *out = e;
    return TT_OK;
}

tt_status tt_engine_destroy(tt_engine* e) {
    if (!e) return TT_OK;
    DeviceGuard dg(e->cfg.device);
    cudaDeviceSynchronize();
    float* fl[] = {e->S_K, e->S_V, e->RW_K, e->RW_V, e->HH_K, e->HH_V, e->HH_scores, e->WR_K, e->WR_V, e->g, e->scratch};
    for (float* p : fl) cudaFree(p);
    cudaFree(e->HH_ids); cudaFree(e->WR_ids); cudaFree(e->ctr); cudaFree(e->job_dev); cudaFree(e->maint_dev);
    cudaFree(e->full_map);
    free_pbs(e);
    delete e;
    return TT_OK;
}

}  // extern "C"

namespace {

// Argument checks shared by the batched and the sharded step.
tt_status validate_step(tt_engine* const* engines, int n, const float* const* Q, const float* const* K_new,
                        const float* const* V_new) {
    if (!engines || !Q || !K_new || !V_new) return set_error(TT_ERR_INVALID_ARGUMENT, "NULL argument.");
    for (int i = 0; i < n; ++i) {
        tt_status s = validate(engines[i]);
        if (s != TT_OK) return s;
        if (!Q[i] || !K_new[i] || !V_new[i])
            return set_error(TT_ERR_INVALID_ARGUMENT, "Q, K_new, V_new and attn_output must not be NULL.");
        const tt_engine_config& a = engines[i]->cfg;
        const tt_engine_config& b = engines[0]->cfg;
        if (a.num_q_heads != b.num_q_heads || a.num_kv_heads != b.num_kv_heads || a.head_dim != b.head_dim ||
            a.device != b.device)
            return set_error(TT_ERR_INVALID_ARGUMENT, "batched engines must share heads, head_dim and device.");
        if (((uintptr_t)Q[i] & 15) || ((uintptr_t)K_new[i] & 15) || ((uintptr_t)V_new[i] & 15))
            return set_error(TT_ERR_INVALID_ARGUMENT, "Q, K_new and V_new must be 16-byte aligned.");
        for (int k = 0; k < i; ++k)
            if (engines[k] == engines[i])
                return set_error(TT_ERR_INVALID_ARGUMENT, "an engine appears more than once in one step.");
    }
    return TT_OK;
}

// Does this step evict a ring token (host mirror of the counters)?
bool step_evicts(const tt_engine* e) { return !(e->h_s < e->cfg.sink_size) && !(e->h_rw < e->cfg.rw_size); }

// Upper bound on the packed blocks after this step's maintenance.
long long step_block_bound(const tt_engine* e) {
    return (e->h_wr_pbs_ub + (step_evicts(e) ? 1 : 0)) / e->chunk;
}

// Maintenance of engines[0..m) in one launch; returns the dense and packed
// token capacities the attention launch must cover.
tt_status maintain_batch(tt_engine* const* engines, int m, const float* const* K_new, const float* const* V_new,
                         cudaStream_t st, int& dcap, int& pcap, const RouteRow* route = nullptr, int world = 1,
                         int route_stride = 0, const unsigned long long* route_flags = nullptr,
                         long long route_step = 0) {
    MaintBatch mb;
    memset(&mb, 0, sizeof(mb));
    mb.n = m;
    mb.route = route;
    mb.world = world;
    mb.route_stride = route_stride > 0 ? route_stride : m;
    mb.route_flags = route_flags;
    mb.route_step = route_step;
    dcap = 0;
    pcap = 0;
    for (int i = 0; i < m; ++i) {
        tt_engine* e = engines[i];
        if (step_evicts(e)) {
            tt_status s = ensure_capacity(e, e->h_wr_pbs_ub + 1);
            if (s != TT_OK) return s;
        }
        mb.d[i] = reinterpret_cast<const MaintDesc*>(e->maint_dev);
        mb.K[i] = K_new[i];
        mb.V[i] = V_new[i];
        dcap = std::max(dcap, dense_cap(e));
        pcap = std::max<long long>(pcap, std::min<long long>(step_block_bound(e), e->pbs_cap) * e->chunk);
    }
    const int ps = prof_begin(0, st);
    k_engine_maintain<<<m, MT, 0, st>>>(mb);
    prof_end(ps, st);
    return check_launch("k_engine_maintain");
}

// Attention launch description for engines[0..m) (jobs, Q, outputs).
void fill_launch(AttnLaunch& L, tt_engine* const* engines, int m, const float* const* Q, float* const* out) {
    L.njobs = m;
    const tt_engine_config& c0 = engines[0]->cfg;
    L.inline_job.hd = c0.head_dim;
    L.inline_job.nq = c0.num_q_heads;
    L.meta_bytes = 2;
    for (int i = 0; i < m; ++i)
        if (!engines[i]->cfg.meta_fp16) L.meta_bytes = 4;
    for (int i = 0; i < m; ++i) {
        L.jobs[i] = engines[i]->job_dev;
        L.Q[i] = Q ? Q[i] : nullptr;
        L.out[i] = out ? out[i] : nullptr;
        L.mw[i] = nullptr;
    }
}

// Host mirrors of the counters after one step of engines[0..m).
void advance_mirrors(tt_engine* const* engines, int m, cudaStream_t st) {
    for (int i = 0; i < m; ++i) {
        tt_engine* e = engines[i];
        if (e->h_s < e->cfg.sink_size) {
            e->h_s++;
        } else if (e->h_rw < e->cfg.rw_size) {
            e->h_rw++;
        } else {
            const int ce = e->h_total - e->cfg.rw_size;  // threshold schedule of k_engine_maintain
            if (ce > e->cfg.sink_size &&
                (e->h_last_calc == -1 || e->h_total - e->h_last_calc >= e->cfg.update_interval))
                e->h_last_calc = e->h_total;
            e->h_rw_head = (e->h_rw_head + 1) % e->cfg.rw_size;
            e->h_evictions++;
            e->h_wr_pbs_ub++;
        }
        e->h_total++;
        e->last_stream = st;
    }
}

// Does the next step of e recompute the heavy-hitter threshold (host mirror
// of k_engine_maintain's schedule)?
bool step_recomputes_threshold(const tt_engine* e) {
    if (!step_evicts(e)) return false;
    return e->h_total - e->cfg.rw_size > e->cfg.sink_size &&
           (e->h_last_calc == -1 || e->h_total - e->h_last_calc >= e->cfg.update_interval);
}

// One rank's share of a sharded launch: at most ceil(n / world) slots of each
// dense tier and ceil(granules / world) packed granules.
void shard_caps(const tt_engine* e, long long blocks, int world, int& dcap_r, int& pcap_r) {
    dcap_r = ceil_div(e->cfg.sink_size, world) + ceil_div(e->max_hh, world) + ceil_div(e->cfg.rw_size, world);
    const long long gran = (std::min<long long>(blocks, e->pbs_cap) * e->chunk + kShardGran - 1) / kShardGran;
    pcap_r = (int)((gran + world - 1) / world) * kShardGran;
}

tt_status validate_shard_args(tt_engine* const* engines, int n, int rank, int world) {
    if (!engines) return set_error(TT_ERR_INVALID_ARGUMENT, "NULL argument.");
    if (n > kMaxBatch) return set_error(TT_ERR_INVALID_ARGUMENT, "a sharded step takes at most %d engines.", kMaxBatch);
    if (world < 1 || world > 64 || rank < 0 || rank >= world)
        return set_error(TT_ERR_INVALID_ARGUMENT, "rank %d / world %d out of range (world <= 64).", rank, world);
    for (int i = 0; i < n; ++i) {
        tt_status s = validate(engines[i]);
        if (s != TT_OK) return s;
    }
    return TT_OK;
}

}  // namespace

extern "C" {

tt_status tt_engine_step_batched(tt_engine* const* engines, int n, const float* const* Q, const float* const* K_new,
                                 const float* const* V_new, float* const* attn_output, void* stream) {
    if (n <= 0) return TT_OK;
    if (!attn_output) return set_error(TT_ERR_INVALID_ARGUMENT, "NULL argument.");
    tt_status s = validate_step(engines, n, Q, K_new, V_new);
    if (s != TT_OK) return s;
    for (int i = 0; i < n; ++i)
        if (!attn_output[i])
            return set_error(TT_ERR_INVALID_ARGUMENT, "Q, K_new, V_new and attn_output must not be NULL.");
    DeviceGuard dg(engines[0]->cfg.device);
    cudaStream_t st = (cudaStream_t)stream;
    for (int base = 0; base < n; base += kMaxBatch) {
        const int m = std::min(kMaxBatch, n - base);
        int dcap = 0, pcap = 0;
        s = maintain_batch(engines + base, m, K_new + base, V_new + base, st, dcap, pcap);
        if (s != TT_OK) return s;
        AttnLaunch L;
        memset(&L, 0, sizeof(L));
        L.njobs = m;
        const tt_engine_config& c0 = engines[base]->cfg;
        s = plan_attention(L, c0.num_q_heads, c0.num_kv_heads, c0.head_dim, dcap, pcap);
        if (s != TT_OK) return s;
        fill_launch(L, engines + base, m, Q + base, attn_output + base);
        L.merge_mode = 1;
        s = launch_attention(L, st);
        if (s != TT_OK) return s;
        advance_mirrors(engines + base, m, st);
    }
    return TT_OK;
}

tt_status tt_engine_sharded_sync_needed(tt_engine* const* engines, int n, int* need) {
    if (!engines || !need) return set_error(TT_ERR_INVALID_ARGUMENT, "NULL argument.");
    *need = 0;
    for (int i = 0; i < n; ++i) {
        tt_status s = validate(engines[i]);
        if (s != TT_OK) return s;
        if (step_recomputes_threshold(engines[i])) *need = 1;
    }
    return TT_OK;
}

tt_status tt_engine_sharded_scores_floats(tt_engine* const* engines, int n, long long* floats) {
    if (!engines || !floats) return set_error(TT_ERR_INVALID_ARGUMENT, "NULL argument.");
    long long t = 0;
    for (int i = 0; i < n; ++i) {
        tt_status s = validate(engines[i]);
        if (s != TT_OK) return s;
        t += engines[i]->cfg.max_seq_len;
    }
    *floats = t;
    return TT_OK;
}

tt_status tt_engine_sharded_scores_pack(tt_engine* const* engines, int n, int rank, int world, float* buf,
                                        void* stream) {
    if (n <= 0) return TT_OK;
    tt_status s = validate_shard_args(engines, n, rank, world);
    if (s != TT_OK) return s;
    if (!buf) return set_error(TT_ERR_INVALID_ARGUMENT, "NULL argument.");
    DeviceGuard dg(engines[0]->cfg.device);
    cudaStream_t st = (cudaStream_t)stream;
    ScoreBatch B;
    memset(&B, 0, sizeof(B));
    B.n = n;
    long long off = 0, items = 1;
    for (int i = 0; i < n; ++i) {
        tt_engine* e = engines[i];
        B.d[i] = reinterpret_cast<const MaintDesc*>(e->maint_dev);
        B.off[i] = off;
        off += e->cfg.max_seq_len;
        items = std::max<long long>(items, (long long)dense_cap(e) + e->chunk + (long long)e->pbs_cap * e->chunk);
    }
    if ((s = check_cuda(cudaMemsetAsync(buf, 0, (size_t)off * sizeof(float), st), "scores pack")) != TT_OK) return s;
    const int gx = (int)std::max<long long>(1, std::min<long long>((items + 255) / 256, std::max(1, 4 * 148 / n)));
    k_scores_pack<<<dim3(gx, n), 256, 0, st>>>(B, rank, world, buf);
    return check_launch("k_scores_pack");
}

tt_status tt_engine_sharded_scores_unpack(tt_engine* const* engines, int n, const float* buf, void* stream) {
    if (n <= 0) return TT_OK;
    if (!engines || !buf) return set_error(TT_ERR_INVALID_ARGUMENT, "NULL argument.");
    if (n > kMaxBatch) return set_error(TT_ERR_INVALID_ARGUMENT, "a sharded step takes at most %d engines.", kMaxBatch);
    for (int i = 0; i < n; ++i) {
        tt_status s = validate(engines[i]);
        if (s != TT_OK) return s;
    }
    DeviceGuard dg(engines[0]->cfg.device);
    cudaStream_t st = (cudaStream_t)stream;
    ScoreBatch B;
    memset(&B, 0, sizeof(B));
    B.n = n;
    long long off = 0, longest = 1;
    for (int i = 0; i < n; ++i) {
        B.d[i] = reinterpret_cast<const MaintDesc*>(engines[i]->maint_dev);
        B.off[i] = off;
        off += engines[i]->cfg.max_seq_len;
        longest = std::max<long long>(longest, engines[i]->cfg.max_seq_len);
    }
    const int gx = (int)std::max<long long>(1, std::min<long long>((longest + 255) / 256, std::max(1, 4 * 148 / n)));
    k_scores_unpack<<<dim3(gx, n), 256, 0, st>>>(B, buf);
    return check_launch("k_scores_unpack");
}

tt_status tt_engine_step_sharded_begin(tt_engine* const* engines, int n, const float* const* Q,
                                       const float* const* K_new, const float* const* V_new, int rank, int world,
                                       const void* route_all, float* xch_send, void* stream) {
    if (n <= 0) return TT_OK;
    tt_status s = validate_shard_args(engines, n, rank, world);
    if (s != TT_OK) return s;
    s = validate_step(engines, n, Q, K_new, V_new);
    if (s != TT_OK) return s;
    if (!xch_send) return set_error(TT_ERR_INVALID_ARGUMENT, "xch_send must not be NULL.");
    if (route_all && ((uintptr_t)route_all & 15))
        return set_error(TT_ERR_INVALID_ARGUMENT, "route_all must be 16-byte aligned.");
    if (route_all && world > 1)
        for (int i = 0; i < n; ++i)
            if (step_recomputes_threshold(engines[i]))
                return set_error(TT_ERR_INVALID_ARGUMENT,
                                 "this step recomputes the heavy-hitter threshold: synchronise the scores "
                                 "(tt_engine_sharded_scores_pack / _unpack) and pass route_all = NULL.");
    DeviceGuard dg(engines[0]->cfg.device);
    cudaStream_t st = (cudaStream_t)stream;
    int dcap = 0, pcap = 0;
    s = maintain_batch(engines, n, K_new, V_new, st, dcap, pcap, static_cast<const RouteRow*>(route_all), world);
    if (s != TT_OK) return s;
    AttnLaunch L;
    memset(&L, 0, sizeof(L));
    L.njobs = n;
    const tt_engine_config& c0 = engines[0]->cfg;
    int dcap_r = 0, pcap_r = 0;
    for (int i = 0; i < n; ++i) {
        int d = 0, p = 0;
        shard_caps(engines[i], step_block_bound(engines[i]), world, d, p);
        dcap_r = std::max(dcap_r, d);
        pcap_r = std::max(pcap_r, p);
    }
    s = plan_attention(L, c0.num_q_heads, c0.num_kv_heads, c0.head_dim, dcap_r, pcap_r);
    if (s != TT_OK) return s;
    // packed chunks cover whole ownership granules (a stage or a 32-token unit
    // never crosses a granule)
    L.PC = ceil_div(L.PC, kShardGran) * kShardGran;
    L.np = ceil_div(pcap_r, L.PC);
    fill_launch(L, engines, n, Q, nullptr);
    L.rank = rank;
    L.world = world;
    L.merge_mode = 1;
    s = launch_sharded_partial(L, xch_send, st);
    if (s != TT_OK) return s;
    advance_mirrors(engines, n, st);
    return TT_OK;
}

tt_status tt_engine_step_sharded_merge(tt_engine* const* engines, int n, int rank, int world, const float* xch_all,
                                       float* const* attn_output, void* route_send, void* stream) {
    if (n <= 0) return TT_OK;
    tt_status s = validate_shard_args(engines, n, rank, world);
    if (s != TT_OK) return s;
    if (!xch_all || !attn_output || !route_send) return set_error(TT_ERR_INVALID_ARGUMENT, "NULL argument.");
    if ((uintptr_t)xch_all & 7) return set_error(TT_ERR_INVALID_ARGUMENT, "xch_all must be 8-byte aligned.");
    if ((uintptr_t)route_send & 15) return set_error(TT_ERR_INVALID_ARGUMENT, "route_send must be 16-byte aligned.");
    for (int i = 0; i < n; ++i)
        if (!attn_output[i]) return set_error(TT_ERR_INVALID_ARGUMENT, "attn_output must not be NULL.");
    DeviceGuard dg(engines[0]->cfg.device);
    AttnLaunch L;
    memset(&L, 0, sizeof(L));
    fill_launch(L, engines, n, nullptr, attn_output);
    L.rank = rank;
    L.world = world;
    int pos_cap = 0;
    for (int i = 0; i < n; ++i) {  // the mirrors already count the step begun
        int d = 0, p = 0;
        shard_caps(engines[i], engines[i]->h_wr_pbs_ub / engines[i]->chunk, world, d, p);
        pos_cap = std::max(pos_cap, d + p);
    }
    return launch_sharded_merge(L, xch_all, static_cast<RouteRow*>(route_send), pos_cap, (cudaStream_t)stream);
}

tt_status tt_sharded_xch_create(int world, int rank, int max_engines, int num_q_heads, int head_dim, int device,
                                tt_xch** out, void* ipc_handle) {
    if (!out || !ipc_handle) return set_error(TT_ERR_INVALID_ARGUMENT, "NULL argument.");
    if (world < 2 || world > kMaxWorld || rank < 0 || rank >= world)
        return set_error(TT_ERR_INVALID_ARGUMENT, "peer exchange needs 2..%d ranks (rank %d of %d).", kMaxWorld, rank,
                         world);
    if (max_engines <= 0 || max_engines > kMaxBatch || num_q_heads <= 0 || head_dim <= 0)
        return set_error(TT_ERR_INVALID_ARGUMENT, "invalid exchange size.");
    DeviceGuard dg(device);
    tt_xch* x = new (std::nothrow) tt_xch();
    if (!x) return set_error(TT_ERR_OUT_OF_MEMORY, "out of host memory.");
    x->world = world; x->rank = rank; x->jobs = max_engines; x->nq = num_q_heads; x->hd = head_dim; x->device = device;
    auto a256 = [](size_t b) { return (b + 255) / 256 * 256; };
    x->rows_bytes = a256((size_t)world * max_engines * num_q_heads * (head_dim + 2) * sizeof(float));
    x->route_bytes = a256((size_t)world * max_engines * sizeof(RouteRow));
    x->flags_bytes = a256((size_t)2 * world * max_engines * sizeof(unsigned long long));
    const size_t total = x->rows_bytes + x->route_bytes + x->flags_bytes;
    tt_status s = check_cuda(cudaMalloc(&x->base, total), "cudaMalloc(exchange region)");
    if (s == TT_OK) s = check_cuda(cudaMemset(x->base, 0, total), "exchange region clear");
    if (s == TT_OK) s = check_cuda(cudaDeviceSynchronize(), "exchange region clear");
    cudaIpcMemHandle_t h;
    if (s == TT_OK) s = check_cuda(cudaIpcGetMemHandle(&h, x->base), "cudaIpcGetMemHandle");
    if (s != TT_OK) {
        if (x->base) cudaFree(x->base);
        delete x;
        return s;
    }
    memcpy(ipc_handle, &h, sizeof(h));
    *out = x;
    return TT_OK;
}

tt_status tt_sharded_xch_open(tt_xch* x, const void* ipc_handles) {
    if (!x || !ipc_handles) return set_error(TT_ERR_INVALID_ARGUMENT, "NULL argument.");
    if (x->opened) return set_error(TT_ERR_INVALID_ARGUMENT, "exchange already opened.");
    DeviceGuard dg(x->device);
    const char* hs = static_cast<const char*>(ipc_handles);
    for (int p = 0; p < x->world; ++p) {
        if (p == x->rank) continue;
        cudaIpcMemHandle_t h;
        memcpy(&h, hs + (size_t)p * sizeof(h), sizeof(h));
        void* ptr = nullptr;
        tt_status s = check_cuda(cudaIpcOpenMemHandle(&ptr, h, cudaIpcMemLazyEnablePeerAccess), "cudaIpcOpenMemHandle");
        if (s != TT_OK) {
            for (int q = 0; q < p; ++q)
                if (x->peer[q]) cudaIpcCloseMemHandle(x->peer[q]);
            return s;
        }
        x->peer[p] = static_cast<char*>(ptr);
    }
    x->opened = true;
    return TT_OK;
}

tt_status tt_sharded_xch_destroy(tt_xch* x) {
    if (!x) return TT_OK;
    DeviceGuard dg(x->device);
    cudaDeviceSynchronize();
    for (int p = 0; p < x->world; ++p)
        if (x->peer[p]) cudaIpcCloseMemHandle(x->peer[p]);
    if (x->base) cudaFree(x->base);
    delete x;
    return TT_OK;
}

namespace {
// The exchange description the kernels get for step x->step.
PeerXch peer_xch(const tt_xch* x) {
    PeerXch px;
    memset(&px, 0, sizeof(px));
    px.world = x->world; px.rank = x->rank; px.jobs = x->jobs; px.step = x->step;
    for (int p = 0; p < x->world; ++p) {
        char* b = p == x->rank ? x->base : x->peer[p];
        px.rows[p] = reinterpret_cast<float*>(b);
        px.route[p] = b + x->rows_bytes;
        px.flags[p] = reinterpret_cast<unsigned long long*>(b + x->rows_bytes + x->route_bytes);
    }
    return px;
}

tt_status validate_xch(const tt_xch* x, tt_engine* const* engines, int n) {
    if (!x || !x->opened) return set_error(TT_ERR_INVALID_ARGUMENT, "exchange not created and opened.");
    if (n > x->jobs) return set_error(TT_ERR_INVALID_ARGUMENT, "%d engines but the exchange holds %d.", n, x->jobs);
    const tt_engine_config& c = engines[0]->cfg;
    if (c.num_q_heads != x->nq || c.head_dim != x->hd || c.device != x->device)
        return set_error(TT_ERR_INVALID_ARGUMENT, "exchange built for other heads, head_dim or device.");
    return TT_OK;
}
}  // namespace

tt_status tt_engine_step_sharded_begin_xch(tt_engine* const* engines, int n, const float* const* Q,
                                           const float* const* K_new, const float* const* V_new, tt_xch* x,
                                           int route_valid, void* stream) {
    if (n <= 0) return TT_OK;
    if (!x) return set_error(TT_ERR_INVALID_ARGUMENT, "NULL argument.");
    tt_status s = validate_shard_args(engines, n, x->rank, x->world);
    if (s != TT_OK) return s;
    if ((s = validate_xch(x, engines, n)) != TT_OK) return s;
    s = validate_step(engines, n, Q, K_new, V_new);
    if (s != TT_OK) return s;
    if (route_valid)
        for (int i = 0; i < n; ++i)
            if (step_recomputes_threshold(engines[i]))
                return set_error(TT_ERR_INVALID_ARGUMENT,
                                 "this step recomputes the heavy-hitter threshold: synchronise the scores "
                                 "(tt_engine_sharded_scores_pack / _unpack) and pass route_valid = 0.");
    if (route_valid && x->step == 0)
        return set_error(TT_ERR_INVALID_ARGUMENT, "no routing rows yet: the first step takes route_valid = 0.");
    DeviceGuard dg(engines[0]->cfg.device);
    cudaStream_t st = (cudaStream_t)stream;
    x->step += 1;
    const PeerXch px = peer_xch(x);
    int dcap = 0, pcap = 0;
    const RouteRow* route = route_valid ? static_cast<const RouteRow*>(px.route[x->rank]) : nullptr;
    s = maintain_batch(engines, n, K_new, V_new, st, dcap, pcap, route, x->world, x->jobs,
                       px.flags[x->rank] + (size_t)x->world * x->jobs, x->step - 1);
    if (s != TT_OK) return s;
    AttnLaunch L;
    memset(&L, 0, sizeof(L));
    L.njobs = n;
    const tt_engine_config& c0 = engines[0]->cfg;
    int dcap_r = 0, pcap_r = 0;
    for (int i = 0; i < n; ++i) {
        int d = 0, p = 0;
        shard_caps(engines[i], step_block_bound(engines[i]), x->world, d, p);
        dcap_r = std::max(dcap_r, d);
        pcap_r = std::max(pcap_r, p);
    }
    s = plan_attention(L, c0.num_q_heads, c0.num_kv_heads, c0.head_dim, dcap_r, pcap_r);
    if (s != TT_OK) return s;
    L.PC = ceil_div(L.PC, kShardGran) * kShardGran;
    L.np = ceil_div(pcap_r, L.PC);
    fill_launch(L, engines, n, Q, nullptr);
    L.rank = x->rank;
    L.world = x->world;
    L.merge_mode = 1;
    L.px = px;
    s = launch_sharded_partial(L, nullptr, st);
    if (s != TT_OK) return s;
    advance_mirrors(engines, n, st);
    return TT_OK;
}

tt_status tt_engine_step_sharded_merge_xch(tt_engine* const* engines, int n, tt_xch* x, float* const* attn_output,
                                           void* stream) {
    if (n <= 0) return TT_OK;
    if (!x || !attn_output) return set_error(TT_ERR_INVALID_ARGUMENT, "NULL argument.");
    tt_status s = validate_shard_args(engines, n, x->rank, x->world);
    if (s != TT_OK) return s;
    if ((s = validate_xch(x, engines, n)) != TT_OK) return s;
    if (x->step == 0) return set_error(TT_ERR_INVALID_ARGUMENT, "merge before the first begin.");
    for (int i = 0; i < n; ++i)
        if (!attn_output[i]) return set_error(TT_ERR_INVALID_ARGUMENT, "attn_output must not be NULL.");
    DeviceGuard dg(engines[0]->cfg.device);
    AttnLaunch L;
    memset(&L, 0, sizeof(L));
    fill_launch(L, engines, n, nullptr, attn_output);
    L.rank = x->rank;
    L.world = x->world;
    L.px = peer_xch(x);
    int pos_cap = 0;
    for (int i = 0; i < n; ++i) {  // the mirrors already count the step begun
        int d = 0, p = 0;
        shard_caps(engines[i], engines[i]->h_wr_pbs_ub / engines[i]->chunk, x->world, d, p);
        pos_cap = std::max(pos_cap, d + p);
    }
    return launch_sharded_merge(L, nullptr, nullptr, pos_cap, (cudaStream_t)stream);
}

tt_status tt_engine_step(tt_engine* e, const float* Q, const float* K_new, const float* V_new, float* attn_output,
                         void* stream) {
    return tt_engine_step_batched(&e, 1, &Q, &K_new, &V_new, &attn_output, stream);
}

tt_status tt_engine_prefill(tt_engine* e, const float* K_all, const float* V_all, int q_len, void* stream) {
    tt_status s = validate(e);
    if (s != TT_OK) return s;
    if (q_len < 0) return set_error(TT_ERR_INVALID_ARGUMENT, "q_len must be non-negative.");
    if (q_len > 0 && (!K_all || !V_all)) return set_error(TT_ERR_INVALID_ARGUMENT, "K_all/V_all must not be NULL.");
    DeviceGuard dg(e->cfg.device);
    cudaStream_t st = (cudaStream_t)stream;
    const int S = e->cfg.sink_size, R = e->cfg.rw_size;
    int nblk = 0;
    if (q_len > S + R) {
        const int n_inter = q_len - R - S;
        nblk = n_inter / e->chunk;
        const int rem = n_inter % e->chunk;
        // WR is overwritten (rem tokens) and nblk blocks are appended
        const long long ub_pbs = (e->h_wr_pbs_ub / e->chunk) * e->chunk + (long long)nblk * e->chunk;
        s = ensure_capacity(e, ub_pbs + rem);
        if (s != TT_OK) return s;
        if (nblk > 0) {
            k_prefill_quantize<<<nblk, 256, 0, st>>>(reinterpret_cast<const MaintDesc*>(e->maint_dev), K_all, V_all);
            if ((s = check_launch("k_prefill_quantize")) != TT_OK) return s;
        }
        e->h_s = S;
        e->h_rw = R;
        e->h_rw_head = 0;
        e->h_evictions += nblk * e->chunk;
        e->h_wr_pbs_ub = ub_pbs + rem;
    } else {
        const int sc = std::min(S, q_len);
        if (sc > 0) e->h_s = sc;
        if (q_len - sc > 0) {
            e->h_rw = q_len - sc;
            e->h_rw_head = 0;
        }
    }
    k_prefill_finish<<<1, 512, 0, st>>>(reinterpret_cast<const MaintDesc*>(e->maint_dev), K_all, V_all, q_len, nblk);
    if ((s = check_launch("k_prefill_finish")) != TT_OK) return s;
    e->h_total = q_len;
    e->last_stream = st;
    return TT_OK;
}

tt_status tt_engine_ingest(tt_engine* e, const float* K_new, const float* V_new, void* stream) {
    tt_status s = validate(e);
    if (s != TT_OK) return s;
    if (!K_new || !V_new) return set_error(TT_ERR_INVALID_ARGUMENT, "K_new and V_new must not be NULL.");
    if (((uintptr_t)K_new & 15) || ((uintptr_t)V_new & 15))
        return set_error(TT_ERR_INVALID_ARGUMENT, "K_new and V_new must be 16-byte aligned.");
    DeviceGuard dg(e->cfg.device);
    cudaStream_t st = (cudaStream_t)stream;
    int dcap = 0, pcap = 0;
    s = maintain_batch(&e, 1, &K_new, &V_new, st, dcap, pcap);
    if (s != TT_OK) return s;
    advance_mirrors(&e, 1, st);
    return TT_OK;
}

tt_status tt_engine_full_count(tt_engine* e, int* count) {
    tt_status s = validate(e);
    if (s != TT_OK) return s;
    if (!count) return set_error(TT_ERR_INVALID_ARGUMENT, "NULL argument.");
    tt_engine_counters c;
    if ((s = tt_engine_get_counters(e, &c)) != TT_OK) return s;
    // live packed tokens: the used blocks' ids other than -1
    DeviceGuard dg(e->cfg.device);
    const size_t np = (size_t)c.pbs_blocks_used * e->chunk;
    long long live = 0;
    if (np > 0) {
        std::vector<int64_t> ids(np);
        if ((s = check_cuda(cudaMemcpy(ids.data(), e->PBS_ids, np * 8, cudaMemcpyDeviceToHost), "ids")) != TT_OK)
            return s;
        for (int64_t v : ids) live += v != -1;
    }
    *count = (int)(c.s_count + c.hh_count + live + c.rw_count);
    return TT_OK;
}

tt_status tt_engine_reconstruct(tt_engine* e, float* K_out, float* V_out, int64_t* ids_out, int capacity,
                                int* count, void* stream) {
    tt_status s = validate(e);
    if (s != TT_OK) return s;
    if (!K_out || !V_out || !ids_out || !count) return set_error(TT_ERR_INVALID_ARGUMENT, "NULL argument.");
    tt_engine_counters c;
    if ((s = tt_engine_get_counters(e, &c)) != TT_OK) return s;
    DeviceGuard dg(e->cfg.device);
    cudaStream_t st = (cudaStream_t)stream;
    const int S = c.s_count, hh = c.hh_count, rw = c.rw_count;
    const long long total = c.total_processed_tokens;
    // middle ids: [S, total - rw) -- every token that left the ring
    const long long lo = S;
    const long long nmid_ids = std::max(0LL, total - rw - lo);
    if (nmid_ids > (1LL << 30)) return set_error(TT_ERR_OUT_OF_RANGE, "token count overflow.");
    const size_t need = (size_t)2 * nmid_ids + 2;  // map [n] + compacted list [n] + count
    if (need > e->full_map_n) {
        cudaFree(e->full_map);
        e->full_map = nullptr;
        e->full_map_n = 0;
        if ((s = dalloc(&e->full_map, need, "full-cache map")) != TT_OK) return s;
        e->full_map_n = need;
    }
    int* map = e->full_map;
    int* list = map + nmid_ids;
    int* dcount = list + nmid_ids + 1;
    const int n = (int)nmid_ids;
    if ((s = check_cuda(cudaMemsetAsync(map, 0xFF, (size_t)n * 4 + 4, st), "map clear")) != TT_OK) return s;
    if ((s = check_cuda(cudaMemsetAsync(dcount, 0, 4, st), "map clear")) != TT_OK) return s;
    const int npbs = c.pbs_blocks_used * e->chunk;
    if (n > 0 && hh + npbs > 0) {
        k_full_map<<<std::max(1, std::min(1184, ceil_div(hh + npbs, 256))), 256, 0, st>>>(
            e->HH_ids, hh, e->PBS_ids, npbs, e->max_hh, lo, n, map);
        if ((s = check_launch("k_full_map")) != TT_OK) return s;
        k_full_compact<<<1, 1024, 0, st>>>(map, n, list, dcount);
        if ((s = check_launch("k_full_compact")) != TT_OK) return s;
    }
    int nmid = 0;
    if ((s = check_cuda(cudaMemcpyAsync(&nmid, dcount, 4, cudaMemcpyDeviceToHost, st), "count")) != TT_OK) return s;
    if ((s = check_cuda(cudaStreamSynchronize(st), "reconstruct")) != TT_OK) return s;
    const int rows = S + nmid + rw;
    *count = rows;
    if (rows > capacity)
        return set_error(TT_ERR_INVALID_ARGUMENT, "capacity %d is below the %d positions of the full cache.",
                         capacity, rows);
    if (rows > 0) {
        const size_t work = (size_t)rows * e->kvs;
        const int grid = (int)std::min<size_t>(148 * 8, (work + 255) / 256);
        k_full_gather<<<std::max(1, grid), 256, 0, st>>>(reinterpret_cast<const MaintDesc*>(e->maint_dev), S, nmid,
                                                         rw, c.rw_head_index, total, lo, map, list, K_out, V_out,
                                                         ids_out);
        if ((s = check_launch("k_full_gather")) != TT_OK) return s;
    }
    e->last_stream = st;
    return TT_OK;
}

tt_status tt_engine_accumulate_scores(tt_engine* e, const float* weights, const int64_t* ids, int n_heads, int n,
                                      void* stream) {
    tt_status s = validate(e);
    if (s != TT_OK) return s;
    if (n < 0 || n_heads <= 0) return set_error(TT_ERR_INVALID_ARGUMENT, "n must be >= 0 and n_heads > 0.");
    if (n == 0) return TT_OK;
    if (!weights) return set_error(TT_ERR_INVALID_ARGUMENT, "weights must not be NULL.");
    DeviceGuard dg(e->cfg.device);
    cudaStream_t st = (cudaStream_t)stream;
    k_accumulate_scores<<<std::max(1, std::min(1184, ceil_div(n, 256))), 256, 0, st>>>(e->g, e->cfg.max_seq_len,
                                                                                     weights, ids, n_heads, n);
    e->last_stream = st;
    return check_launch("k_accumulate_scores");
}

tt_status tt_engine_get_counters(tt_engine* e, tt_engine_counters* out) {
    tt_status s = validate(e);
    if (s != TT_OK) return s;
    if (!out) return set_error(TT_ERR_INVALID_ARGUMENT, "NULL argument.");
    DeviceGuard dg(e->cfg.device);
    if ((s = check_cuda(cudaStreamSynchronize(e->last_stream), "engine sync")) != TT_OK) return s;
    DevCounters c;
    if ((s = check_cuda(cudaMemcpy(&c, e->ctr, sizeof(c), cudaMemcpyDeviceToHost), "counter read")) != TT_OK) return s;
    if (c.error)
        return set_error((tt_status)c.error, "device-side engine error %d (%s)", c.error,
                         c.error == TT_ERR_TIMEOUT ? "a bounded wait ran out" : "packed capacity");
    out->s_count = c.s_count;
    out->rw_count = c.rw_count;
    out->rw_head_index = c.rw_head;
    out->hh_count = c.hh_count;
    out->wr_count = c.wr_count;
    out->pbs_allocated_blocks = c.pbs_alloc;
    out->pbs_blocks_used = c.pbs_used;
    out->pbs_count = c.pbs_count;
    out->total_processed_tokens = c.total;
    out->total_evictions = c.total_evictions;
    out->last_calc_pos = c.last_calc_pos;
    out->max_hh = e->max_hh;
    out->chunk_size = e->chunk;
    out->cached_threshold = c.cached_threshold;
    return TT_OK;
}

tt_status tt_engine_set_counters(tt_engine* e, const tt_engine_counters* in, void* stream) {
    tt_status s = validate(e);
    if (s != TT_OK) return s;
    if (!in) return set_error(TT_ERR_INVALID_ARGUMENT, "NULL argument.");
    const tt_engine_counters& c = *in;
    if (c.s_count < 0 || c.s_count > e->cfg.sink_size || c.rw_count < 0 || c.rw_count > e->cfg.rw_size ||
        c.rw_head_index < 0 || c.rw_head_index >= e->cfg.rw_size || c.hh_count < 0 || c.hh_count > e->max_hh ||
        c.wr_count < 0 || c.wr_count >= e->chunk || c.pbs_blocks_used < 0 ||
        c.pbs_allocated_blocks < c.pbs_blocks_used || c.pbs_count != c.pbs_blocks_used * e->chunk ||
        c.total_processed_tokens < 0)
        return set_error(TT_ERR_INVALID_ARGUMENT, "inconsistent engine counters.");
    DeviceGuard dg(e->cfg.device);
    if (std::max(c.pbs_blocks_used + 1 + kLogicalSlack, c.pbs_allocated_blocks) > e->pbs_cap) {
        if ((s = grow_pbs(e, std::max(c.pbs_blocks_used + 1 + kLogicalSlack, c.pbs_allocated_blocks))) != TT_OK)
            return s;
    }
    DevCounters d;
    memset(&d, 0, sizeof(d));
    d.s_count = c.s_count; d.rw_count = c.rw_count; d.rw_head = c.rw_head_index; d.hh_count = c.hh_count;
    d.wr_count = c.wr_count; d.pbs_alloc = c.pbs_allocated_blocks; d.pbs_used = c.pbs_blocks_used;
    d.pbs_count = c.pbs_count; d.total = c.total_processed_tokens; d.total_evictions = c.total_evictions;
    d.last_calc_pos = c.last_calc_pos; d.cached_threshold = c.cached_threshold;
    cudaStream_t st = (cudaStream_t)stream;
    if ((s = check_cuda(cudaMemcpyAsync(e->ctr, &d, sizeof(d), cudaMemcpyHostToDevice, st), "set counters")) != TT_OK)
        return s;
    if ((s = check_cuda(cudaStreamSynchronize(st), "set counters")) != TT_OK) return s;
    e->h_total = c.total_processed_tokens;
    e->h_s = c.s_count;
    e->h_rw = c.rw_count;
    e->h_rw_head = c.rw_head_index;
    e->h_evictions = c.total_evictions;
    e->h_last_calc = c.last_calc_pos;
    e->h_wr_pbs_ub = (long long)c.pbs_count + c.wr_count;
    e->last_stream = st;
    return TT_OK;
}

tt_status tt_engine_get_buffer(tt_engine* e, int which, tt_buffer_desc* out) {
    tt_status s = validate(e);
    if (s != TT_OK) return s;
    if (!out) return set_error(TT_ERR_INVALID_ARGUMENT, "NULL argument.");
    tt_engine_counters c;
    if ((s = tt_engine_get_counters(e, &c)) != TT_OK) return s;
    const size_t kvs = e->kvs, nb = (size_t)c.pbs_allocated_blocks, C = e->chunk;
    const int m16 = e->cfg.meta_fp16;
    const int mdt = m16 ? 3 : 0, mes = m16 ? 2 : 4;
    auto set = [&](void* p, size_t n, int es, int dt) {
        out->data = p; out->count = n; out->elem_size = es; out->dtype = dt;
        return TT_OK;
    };
    switch (which) {
        case TT_BUF_S_K: return set(e->S_K, (size_t)e->cfg.sink_size * kvs, 4, 0);
        case TT_BUF_S_V: return set(e->S_V, (size_t)e->cfg.sink_size * kvs, 4, 0);
        case TT_BUF_RW_K: return set(e->RW_K, (size_t)e->cfg.rw_size * kvs, 4, 0);
        case TT_BUF_RW_V: return set(e->RW_V, (size_t)e->cfg.rw_size * kvs, 4, 0);
        case TT_BUF_HH_K: return set(e->HH_K, (size_t)e->max_hh * kvs, 4, 0);
        case TT_BUF_HH_V: return set(e->HH_V, (size_t)e->max_hh * kvs, 4, 0);
        case TT_BUF_HH_TOKEN_IDS: return set(e->HH_ids, (size_t)e->max_hh, 8, 2);
        case TT_BUF_HH_SCORES: return set(e->HH_scores, (size_t)e->max_hh, 4, 0);
        case TT_BUF_WR_K: return set(e->WR_K, C * kvs, 4, 0);
        case TT_BUF_WR_V: return set(e->WR_V, C * kvs, 4, 0);
        case TT_BUF_WR_TOKEN_IDS: return set(e->WR_ids, C, 8, 2);
        case TT_BUF_PBS_K_PACKED: return set(e->kp, nb * (C / 16) * kvs, 4, 1);
        case TT_BUF_PBS_K_SCALES: return set(e->ks, nb * kvs, mes, mdt);
        case TT_BUF_PBS_K_ZEROES: return set(e->kz, nb * kvs, mes, mdt);
        case TT_BUF_PBS_V_PACKED: return set(e->vp, nb * C * e->cfg.num_kv_heads * e->qhd, 4, 1);
        case TT_BUF_PBS_V_SCALES: return set(e->vs, nb * C * e->cfg.num_kv_heads, mes, mdt);
        case TT_BUF_PBS_V_ZEROES: return set(e->vz, nb * C * e->cfg.num_kv_heads, mes, mdt);
        case TT_BUF_PBS_TOKEN_IDS: return set(e->PBS_ids, nb * C, 8, 2);
        case TT_BUF_GLOBAL_ATTN_SCORES: return set(e->g, (size_t)e->cfg.max_seq_len, 4, 0);
    }
    return set_error(TT_ERR_OUT_OF_RANGE, "unknown buffer id %d", which);
}

tt_status tt_engine_get_buffer_bytes(tt_engine* e, size_t* out) {
    tt_status s = validate(e);
    if (s != TT_OK) return s;
    tt_engine_counters c;
    if ((s = tt_engine_get_counters(e, &c)) != TT_OK) return s;
    // cache_engine.cpp:543-568 over the reference's logical sizes
    const size_t kvs = e->kvs, nb = (size_t)c.pbs_allocated_blocks, C = e->chunk, mb = e->meta_bytes;
    size_t b = 0;
    b += 2 * (size_t)e->cfg.sink_size * kvs * 4 + 2 * (size_t)e->cfg.rw_size * kvs * 4;
    b += 2 * (size_t)e->max_hh * kvs * 4 + (size_t)e->max_hh * 8 + (size_t)e->max_hh * 4;
    b += 2 * C * kvs * 4 + C * 8;
    b += nb * (C / 16) * kvs * 4;
    b += 2 * nb * kvs * mb + 2 * nb * C * e->cfg.num_kv_heads * mb;
    b += nb * C * e->cfg.num_kv_heads * e->qhd * 4 + nb * C * 8;
    b += (size_t)e->cfg.max_seq_len * 4;
    *out = b;
    return TT_OK;
}

tt_status tt_engine_device_bytes(tt_engine* e, size_t* out) {
    tt_status s = validate(e);
    if (s != TT_OK) return s;
    const size_t kvs = e->kvs, nb = (size_t)e->pbs_cap, C = e->chunk, mb = e->meta_bytes;
    size_t b = 0;
    b += 2 * (size_t)std::max(e->cfg.sink_size, 1) * kvs * 4 + 2 * (size_t)e->cfg.rw_size * kvs * 4;
    b += 2 * (size_t)e->max_hh * kvs * 4 + (size_t)e->max_hh * 12 + 2 * C * kvs * 4 + C * 8;
    b += nb * (C / 16) * kvs * 4 + 2 * nb * kvs * mb + 2 * nb * C * e->cfg.num_kv_heads * mb;
    b += nb * C * e->cfg.num_kv_heads * e->qhd * 4 + nb * C * 8 + (size_t)e->cfg.max_seq_len * 4;
    b += e->scratch_floats * 4 + sizeof(DevCounters) + sizeof(JobDesc) + sizeof(MaintDesc);
    *out = b;
    return TT_OK;
}

}  // extern "C"
