// tt_attn.cu -- fused single-query decode attention over the tiered KV cache.
//
// Replaces the reference's fused_attention_decode_avx2
// (csrc/cpu/fused_attn_avx2.cpp:145-301), which dequantizes the whole packed
// background store (PBS) into scratch, materialises an nq x T score matrix
// and walks it per query head.  Here the work is split-KV:
//
//   k_attn_dense   grid = (dense chunks, jobs x kv-head groups), 8 warps
//     (tt_dense.cuh).  The FP32 sink / heavy-hitter / ring rows staged by 1-D
//     TMA bulk copies: QK with the G query heads of each kv head (GQA: every
//     K byte is read once), online softmax in log2 units, PV.
//   k_attn_packed  grid = (packed chunks, jobs x kv-head groups), 8 warps
//     (tt_partial.cuh).  2-bit codes used in place as 4 + code (tensor-core
//     unit, tt_pbs_mma.cuh, or the SIMT unit): score = sum(q*scale*(4+code))
//     - 4 sum(q*scale) + sum(q*zero), no dequantized copy; the per-token V
//     scale folded into the weight, the zero into a running sum.
//   The two run concurrently (the dense one on a second stream, forked and
//   joined with events): the memory-bound dense chunks and the issue-bound
//   packed chunks share the SMs.  Output: per (chunk, q head) partial
//   (m, l, acc[hd]) and the raw logits (for the mean attention weights).
//   For engine steps the last CTA of each job, of either kernel, merges the
//   job's chunk partials (log-sum-exp) into attn_output and the heads'
//   (M, 1/L) -- or, sequence-sharded, into the job's exchange row.
//   k_attn_merge_heads grid = (q heads, jobs, groups).  The same merge for
//     stand-alone calls and jobs with more than 128 chunk slots (two passes
//     above 64 slots).
//   k_attn_weights grid = (one wave of CTAs over the launch, jobs), CTAs
//     striding over positions, four per thread.  The head-mean softmax
//     weights (fused_attn_avx2.cpp:286-300) and, for engine jobs, the decayed
//     score feedback g[id] = decay*g[id] + w (cache_engine.cpp:511-540).
//   k_shard_merge (sequence-sharded steps) grid = (one wave of CTAs, jobs).
//     Every rank's rows -> output, the feedback of this rank's own tokens and
//     the job's routing row; with the peer exchange it first waits for the
//     other ranks' rows in its own memory.
#include <algorithm>
#include <climits>
#include <mutex>

#include "tt_attn.cuh"

#include "tt_partial.cuh"
#include "tt_dense.cuh"

namespace tt {

// ---------------------------------------------------------------------------
// merge + mean weights + score feedback
// ---------------------------------------------------------------------------
// Merge of one head's chunk partials: M = max m, L = sum l 2^(m - M),
// out = sum acc 2^(m - M) / L (row_sum_exp fallback, fused_attn_avx2.cpp:261).
// grid (nq, njobs, groups); warps split the chunks; dynamic shared memory:
// (group + 1 + NW * hd) floats.  Jobs with many chunks merge in two passes:
// pass 1 (final = 0) merges each group of `group` chunks into the group's
// first slot, unnormalised; pass 2 (final = 1, stride = that group size)
// merges the group results at slots 0, stride, 2 stride, ...
__global__ void __launch_bounds__(NT) k_attn_merge_heads(const __grid_constant__ AttnLaunch L, int group, int stride,
                                                         int final_pass) {
    extern __shared__ float fsm[];
    __shared__ JobDesc Js;
    __shared__ TierCounts Ts;
    __shared__ float red[NW];
    __shared__ float Mh, Lh;
    const int job = blockIdx.y, h = blockIdx.x;
    if (threadIdx.x == 0) {
        Js = L.jobs[job] ? *L.jobs[job] : L.inline_job;
        Ts = resolve_counts(Js);
    }
    __syncthreads();
    const JobDesc& J = Js;
    const TierCounts tc = Ts;
    const int nq = J.nq, HD = J.hd;
    const int D = tc.n0 + tc.n1 + tc.n2;
    const int nd_act = ceil_div(D, L.DC), np_act = ceil_div(tc.nblk * J.grp, L.PC);
    const int nch_all = ceil_div(nd_act + np_act, stride);  // entries of this pass
    const int c0 = blockIdx.z * group;
    const int nch = max(0, min(group, nch_all - c0));
    if (!final_pass && nch == 0) return;
    float* wts = fsm;                        // [group]
    float* acc = fsm + group + 1;            // [NW][HD]
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    // compact partial slots (dense chunks first), every stride-th in pass 2
    auto chunk_index = [&](int i) { return (c0 + i) * stride; };

    float M = -INFINITY;
    for (int i = threadIdx.x; i < nch; i += NT) M = fmaxf(M, J.part_ml[((size_t)chunk_index(i) * nq + h) * 2]);
    M = warp_max(M);
    if (lane == 0) red[warp] = M;
    __syncthreads();
    if (threadIdx.x == 0) {
        float m = red[0];
        for (int w = 1; w < NW; ++w) m = fmaxf(m, red[w]);
        Mh = m;
    }
    __syncthreads();
    M = Mh;
    float S = 0.f;
    for (int i = threadIdx.x; i < nch; i += NT) {
        const size_t pi = ((size_t)chunk_index(i) * nq + h) * 2;
        const float mi = J.part_ml[pi];
        const float w = (M == -INFINITY || mi == -INFINITY) ? 0.f : exp2f(mi - M);
        wts[i] = w;
        S = fmaf(J.part_ml[pi + 1], w, S);
    }
    S = warp_sum(S);
    __syncthreads();
    if (lane == 0) red[warp] = S;
    __syncthreads();
    if (threadIdx.x == 0) {
        float t = 0.f;
        for (int w = 0; w < NW; ++w) t += red[w];
        Lh = t;
    }
    __syncthreads();
    // each warp sums a strided subset of the chunks over all channels
    for (int c = lane; c < HD; c += 32) {
        float o = 0.f;
#pragma unroll 4
        for (int i = warp; i < nch; i += NW) o = fmaf(J.part_acc[((size_t)chunk_index(i) * nq + h) * HD + c], wts[i], o);
        acc[warp * HD + c] = o;
    }
    __syncthreads();  // every read of this group's slots is done before the first slot is overwritten
    if (!final_pass) {
        const size_t pi = (size_t)chunk_index(0) * nq + h;
        for (int c = threadIdx.x; c < HD; c += NT) {
            float t = 0.f;
            for (int w = 0; w < NW; ++w) t += acc[w * HD + c];
            J.part_acc[pi * HD + c] = t;
        }
        if (threadIdx.x == 0) {
            J.part_ml[pi * 2] = M;
            J.part_ml[pi * 2 + 1] = Lh;
        }
        return;
    }
    const float inv = 1.0f / (Lh > 0.f ? Lh : 1.0f);
    float* out = L.out[job];
    for (int c = threadIdx.x; c < HD; c += NT) {
        float t = 0.f;
        for (int w = 0; w < NW; ++w) t += acc[w * HD + c];
        out[(size_t)h * HD + c] = t * inv;
    }
    if (threadIdx.x == 0) {
        float* ml = head_ml(J);
        ml[2 * h] = M;
        ml[2 * h + 1] = inv;
    }
}

// Mean attention weights over heads (fused_attn_avx2.cpp:286-300) and, for
// engines, the score feedback.  Four consecutive positions per thread (float4
// logit rows; the token ids and old scores are loaded first, so their latency
// overlaps the logit loads), CTAs striding over the job's positions; one
// position per thread where the logit rows are not 16-byte aligned.
// grid (gx, njobs); dynamic shared memory: 2 nq floats.
__global__ void __launch_bounds__(NT, 4) k_attn_weights(const __grid_constant__ AttnLaunch L) {
    extern __shared__ float fsm[];
    __shared__ JobDesc Js;
    __shared__ TierCounts Ts;
    const int job = blockIdx.y;
    if (threadIdx.x == 0) Js = L.jobs[job] ? *L.jobs[job] : L.inline_job;
    __syncthreads();
    const JobDesc& J = Js;
    const int nq = J.nq;
    float* Ms = fsm;
    float* IL = fsm + nq;
    // the heads' (M, 1/L) and the tier counters are independent loads: one round trip
    if (threadIdx.x == 0) Ts = resolve_counts(J);
    const float* ml = head_ml(J);
    for (int h = threadIdx.x; h < nq; h += NT) {
        const float m = ml[2 * h];
        Ms[h] = m == -INFINITY ? INFINITY : m;  // a head without logits: every term 2^-inf = 0
        IL[h] = ml[2 * h + 1];
    }
    __syncthreads();
    const TierCounts tc = Ts;
    const int D = tc.n0 + tc.n1 + tc.n2;
    const int T = D + tc.nblk * J.grp;
    float* mw = L.mw[job];
    const bool vec = ((reinterpret_cast<uintptr_t>(J.scores) & 15) == 0) && (J.score_stride & 3) == 0;
    if (!vec) {
        for (int pos = blockIdx.x * NT + threadIdx.x; pos < T; pos += gridDim.x * NT)
            weigh_position(J, tc, D, Ms, IL, mw, pos);
        return;
    }
    for (int p4 = (blockIdx.x * NT + threadIdx.x) * 4; p4 < T; p4 += gridDim.x * NT * 4) {
        long long id[4];
        int hh[4];
        float g0[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            hh[k] = -1;
            id[k] = (J.g && p4 + k < T) ? position_id(J, tc, D, p4 + k, hh[k]) : -1;
            if (id[k] >= J.msl) id[k] = -1;
        }
#pragma unroll
        for (int k = 0; k < 4; ++k) g0[k] = id[k] >= 0 ? J.g[id[k]] : 0.f;
        const float4 w4 = mean_weight4(J, Ms, IL, nq, p4);  // rows are stride >= T + 3 floats long
        const float w[4] = {w4.x, w4.y, w4.z, w4.w};
        if (mw) {
#pragma unroll
            for (int k = 0; k < 4; ++k)
                if (p4 + k < T) mw[p4 + k] = w[k];
        }
#pragma unroll
        for (int k = 0; k < 4; ++k) {  // positions hold distinct tokens: no two updates meet
            if (id[k] < 0) continue;
            const float nv = fmaf(J.decay, g0[k], w[k]);
            J.g[id[k]] = nv;
            if (hh[k] >= 0) J.hh_scores[hh[k]] = nv;
        }
    }
}

// ---------------------------------------------------------------------------
// sequence-sharded attention (see launch_sharded_* in tt_attn.cuh)
// ---------------------------------------------------------------------------
// Phase 1 epilogue for launches with many chunk slots: this rank's chunk
// partials -> one (m, l, acc) row per head.  grid (nq, njobs); dynamic shared
// memory: nd + np + 1 floats.
__global__ void __launch_bounds__(NT) k_shard_local_merge(const __grid_constant__ AttnLaunch L, float* xch) {
    extern __shared__ float wts[];
    __shared__ JobDesc Js;
    __shared__ TierCounts Ts;
    __shared__ float red[NW];
    __shared__ float Mh, Lh;
    const int job = blockIdx.y, h = blockIdx.x;
    if (threadIdx.x == 0) {
        Js = L.jobs[job] ? *L.jobs[job] : L.inline_job;
        Ts = resolve_counts(Js);
    }
    __syncthreads();
    const JobDesc& J = Js;
    const TierCounts tc = Ts;
    const int nq = J.nq, HD = J.hd;
    const ShardMap SM = shard_map(tc, J.grp, L.rank, L.world);
    const int nch = ceil_div(SM.nd, L.DC) + ceil_div(SM.np, L.PC);  // compact partial slots, dense chunks first
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    float M = -INFINITY;
    for (int i = threadIdx.x; i < nch; i += NT) M = fmaxf(M, J.part_ml[((size_t)i * nq + h) * 2]);
    M = warp_max(M);
    if (lane == 0) red[warp] = M;
    __syncthreads();
    if (threadIdx.x == 0) {
        float m = red[0];
        for (int w = 1; w < NW; ++w) m = fmaxf(m, red[w]);
        Mh = m;
    }
    __syncthreads();
    M = Mh;
    float S = 0.f;
    for (int i = threadIdx.x; i < nch; i += NT) {
        const size_t pi = ((size_t)i * nq + h) * 2;
        const float mi = J.part_ml[pi];
        const float w = (M == -INFINITY || mi == -INFINITY) ? 0.f : exp2f(mi - M);
        wts[i] = w;
        S = fmaf(J.part_ml[pi + 1], w, S);
    }
    S = warp_sum(S);
    __syncthreads();
    if (lane == 0) red[warp] = S;
    __syncthreads();
    if (threadIdx.x == 0) {
        float t = 0.f;
        for (int w = 0; w < NW; ++w) t += red[w];
        Lh = t;
    }
    __syncthreads();
    float* dst = xch + ((size_t)job * nq + h) * (HD + 2);
    for (int c = threadIdx.x; c < HD; c += NT) {
        float o = 0.f;
        for (int i = 0; i < nch; ++i) o = fmaf(J.part_acc[((size_t)i * nq + h) * HD + c], wts[i], o);
        dst[2 + c] = o;
    }
    if (threadIdx.x == 0) {
        dst[0] = M;
        dst[1] = Lh;
        if (h == 0) *route_min_word(J) = 0ull;
    }
}

// Peer exchange after k_shard_local_merge: this rank's rows of job
// blockIdx.x, already in its own region's slot, copied into every other
// rank's region, then the job's flag set on every rank.  grid (njobs).
__global__ void __launch_bounds__(NT) k_publish_rows(const __grid_constant__ AttnLaunch L) {
    const int job = blockIdx.x;
    const int nq = L.inline_job.nq, HD = L.inline_job.hd;
    const size_t n = (size_t)nq * (HD + 2), off = ((size_t)L.px.rank * L.px.jobs + job) * n;
    const float* src = L.px.rows[L.px.rank] + off;
    for (int p = 0; p < L.px.world; ++p) {
        if (p == L.px.rank) continue;
        float* dst = L.px.rows[p] + off;
        for (size_t i = threadIdx.x; i < n; i += NT) dst[i] = src[i];
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence_system();
        for (int p = 0; p < L.px.world; ++p)
            st_release_sys(L.px.flags[p] + (size_t)L.px.rank * L.px.jobs + job, (unsigned long long)L.px.step);
    }
}

// Phase 2: every rank's rows -> output (ranks merged in order 0..world-1, so
// all ranks produce the same bits), the decayed score feedback
// g[id] = decay g[id] + w of the tokens this rank owns (cache_engine.cpp:
// 511-540; only the owner keeps a token's score current), and the job's
// routing row from its last CTA.  grid (gx, njobs); dynamic shared memory:
// 2 nq floats.
__global__ void __launch_bounds__(NT, 3) k_shard_merge(const __grid_constant__ AttnLaunch L, const float* xch_all,
                                                    RouteRow* route) {
    extern __shared__ float sm[];
    __shared__ JobDesc Js;
    __shared__ TierCounts Ts;
    __shared__ unsigned long long red_key[NW];
    const int job = blockIdx.y;
    if (threadIdx.x == 0) Js = L.jobs[job] ? *L.jobs[job] : L.inline_job;
    __syncthreads();
    const JobDesc& J = Js;
    const bool peer = L.px.world > 1;
    if (threadIdx.x == 0) {
        Ts = resolve_counts(J);
        // peer exchange: every rank's rows of this job have landed in this
        // rank's region (bounded wait; on expiry the error is recorded and
        // the step's results are not valid)
        if (peer && !wait_peer_flags(L.px.flags[L.px.rank] + job, L.px.jobs, L.px.world, L.px.step)) {
            atomicCAS(&g_device_error, 0, (int)TT_ERR_TIMEOUT);
            if (J.ctr) atomicCAS(const_cast<int*>(&J.ctr->error), 0, (int)TT_ERR_TIMEOUT);
        }
    }
    __syncthreads();
    const int nq = J.nq, HD = J.hd, P = L.world;
    float* Ms = sm;
    float* IL = sm + nq;
    const size_t row = (size_t)HD + 2, rstride = (size_t)(peer ? L.px.jobs : L.njobs) * nq * row;
    const float* base = (peer ? L.px.rows[L.px.rank] : xch_all) + (size_t)job * nq * row;
    // (M, 1/L) of every head: 8 adjacent threads per head, each holding the
    // (m, l) pairs of ranks sub, sub + 8, ... (one load round for P <= 8)
    for (int h0 = 0; h0 < nq; h0 += NT / 8) {
        const int h = h0 + threadIdx.x / 8, sub = threadIdx.x % 8;
        constexpr int PR = 4;  // ranks per thread held in registers (P <= 32)
        float2 ml[PR];
#pragma unroll
        for (int k = 0; k < PR; ++k) {
            const int p = sub + 8 * k;
            ml[k] = (h < nq && p < P) ? *reinterpret_cast<const float2*>(base + p * rstride + h * row)
                                      : make_float2(-INFINITY, 0.f);
        }
        float M = -INFINITY;
#pragma unroll
        for (int k = 0; k < PR; ++k) M = fmaxf(M, ml[k].x);
        for (int p = sub + 8 * PR; p < P && h < nq; p += 8) M = fmaxf(M, base[p * rstride + h * row]);
#pragma unroll
        for (int x = 1; x < 8; x <<= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, x));
        float S = 0.f;
        if (M != -INFINITY) {
#pragma unroll
            for (int k = 0; k < PR; ++k)
                if (ml[k].x != -INFINITY) S = fmaf(ml[k].y, exp2f(ml[k].x - M), S);
            for (int p = sub + 8 * PR; p < P && h < nq; p += 8) {
                const float mp = base[p * rstride + h * row];
                if (mp != -INFINITY) S = fmaf(base[p * rstride + h * row + 1], exp2f(mp - M), S);
            }
        }
#pragma unroll
        for (int x = 1; x < 8; x <<= 1) S += __shfl_xor_sync(0xffffffffu, S, x);
        if (sub == 0 && h < nq) {
            Ms[h] = M;
            IL[h] = 1.0f / (S > 0.f ? S : 1.0f);
        }
    }
    __syncthreads();
    const TierCounts tc = Ts;
    float* out = L.out[job];
    // the job's nq x hd outputs spread over its CTAs, one (head, channel) per
    // thread and pass, so that a few CTAs cover them
    for (int i = blockIdx.x * NT + threadIdx.x; i < nq * HD; i += gridDim.x * NT) {
        const int h = i / HD, c = i - h * HD;
        const float M = Ms[h], inv = IL[h];
        float o = 0.f;
        for (int p = 0; p < P; ++p) {
            const float mp = base[p * rstride + h * row];
            if (M != -INFINITY && mp != -INFINITY)
                o = fmaf(base[p * rstride + h * row + 2 + c], exp2f(mp - M) * inv, o);
        }
        out[(size_t)h * HD + c] = o;
    }
    __syncthreads();  // every thread has read Ms before the substitution below
    for (int h = threadIdx.x; h < nq; h += NT)
        if (Ms[h] == -INFINITY) Ms[h] = INFINITY;  // a head without logits: every term 2^-inf = 0
    __syncthreads();
    // feedback of this rank's positions; the heavy-hitter minimum over them
    const int r = L.rank;
    const ShardMap SM = shard_map(tc, J.grp, r, P);
    const int n_loc = SM.nd + SM.np;
    unsigned long long best = 0ull;  // complemented key, 0 = none
    const bool vec = ((reinterpret_cast<uintptr_t>(J.scores) & 15) == 0) && (J.score_stride & 3) == 0;
    if (J.g) {
        const int per = vec ? 4 : 1;  // positions per thread: float4 logit rows where aligned
        for (int i0 = (blockIdx.x * NT + threadIdx.x) * per; i0 < n_loc; i0 += gridDim.x * NT * per) {
            long long id[4];
            int hh[4];
            float g0[4], w[4];
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                hh[k] = -1;
                id[k] = (k < per && i0 + k < n_loc) ? local_position_id(J, tc, SM, r, P, i0 + k, hh[k]) : -1;
                if (id[k] >= J.msl) id[k] = -1;
            }
#pragma unroll
            for (int k = 0; k < 4; ++k) g0[k] = id[k] >= 0 ? J.g[id[k]] : 0.f;
            if (vec) {
                const float4 w4 = mean_weight4(J, Ms, IL, nq, i0);
                w[0] = w4.x; w[1] = w4.y; w[2] = w4.z; w[3] = w4.w;
            } else {
                w[0] = mean_weight(J, Ms, IL, nq, i0);
                w[1] = w[2] = w[3] = 0.f;
            }
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                if (id[k] < 0) continue;
                const float nv = fmaf(J.decay, g0[k], w[k]);
                J.g[id[k]] = nv;
                if (hh[k] >= 0) {
                    J.hh_scores[hh[k]] = nv;
                    const unsigned long long key = ~(((unsigned long long)order_key(nv) << 32) | (uint32_t)hh[k]);
                    best = key > best ? key : best;
                }
            }
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const unsigned long long v = __shfl_xor_sync(0xffffffffu, best, o);
        best = v > best ? v : best;
    }
    if ((threadIdx.x & 31) == 0) red_key[threadIdx.x >> 5] = best;
    __shared__ int last;
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int w = 1; w < NW; ++w) best = red_key[w] > best ? red_key[w] : best;
        if (best) atomicMax(route_min_word(J), best);
        __threadfence();
        last = atomicAdd(job_counter(J), 1) == (int)gridDim.x - 1;
        if (last) {
            __threadfence();
            const unsigned long long k = atomicExch(route_min_word(J), 0ull);
            RouteRow rr;
            rr.ev_score = 0.f;
            rr.hh_min = 0.f;
            rr.hh_slot = -1;
            rr.pad = 0;
            if (k) {
                const unsigned long long key = ~k;
                rr.hh_min = key_value((uint32_t)(key >> 32));
                rr.hh_slot = (int)(uint32_t)key;
            }
            // the token the next step evicts: ring slot ring_head, id total - R
            if (J.g && tc.ring_size > 0 && tc.n2 == tc.ring_size && tc.ring_head % P == r) {
                const long long id = (long long)tc.total - tc.ring_size;
                if (id >= 0 && id < J.msl) rr.ev_score = __ldcg(J.g + id);
            }
            if (peer) {  // into every rank's region at this rank's slot, then the flags
                for (int p = 0; p < L.px.world; ++p)
                    reinterpret_cast<RouteRow*>(L.px.route[p])[(size_t)L.px.rank * L.px.jobs + job] = rr;
                __threadfence_system();
                for (int p = 0; p < L.px.world; ++p)
                    st_release_sys(L.px.flags[p] + (size_t)(L.px.world + L.px.rank) * L.px.jobs + job,
                                   (unsigned long long)L.px.step);
            } else {
                route[job] = rr;
            }
            *job_counter(J) = 0;
        }
    }
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
int attn_max_chunks(int dense_cap, int pbs_tok_cap) { return ceil_div(dense_cap, 32) + ceil_div(pbs_tok_cap, 64) + 2; }

static int pick_gm(int G) {
    if (G <= 1) return 1;
    if (G <= 2) return 2;
    if (G <= 4) return 4;
    if (G <= 8) return 8;
    return 0;
}

tt_status plan_attention(AttnLaunch& L, int nq, int nkv, int hd, int dense_cap, int pbs_tok_cap) {
    if (nkv <= 0 || nq % nkv != 0) return set_error(TT_ERR_UNSUPPORTED, "num_q_heads must be a multiple of num_kv_heads.");
    L.G = nq / nkv;
    if (!pick_gm(L.G)) return set_error(TT_ERR_UNSUPPORTED, "more than 8 query heads per kv head is not supported.");
    if (hd != 16 && hd != 32 && hd != 64 && hd != 128 && hd != 256)
        return set_error(TT_ERR_UNSUPPORTED, "head_dim %d not supported (16, 32, 64, 128, 256).", hd);
    // A kv-head group is staged as one contiguous run per region when it holds
    // every kv head (nkv <= 8); wider models split into groups of 8.
    if (L.G > 4 && nkv % 4 == 0) {
        L.HG = 4;  // the tensor-core unit runs 5..8 query heads as two warps per kv head
    } else if (nkv <= 8) {
        L.HG = nkv;
    } else if (nkv % 8 == 0) {
        L.HG = 8;
    } else {
        return set_error(TT_ERR_UNSUPPORTED, "num_kv_heads > 8 must be a multiple of 8 (got %d).", nkv);
    }
    L.nhg = nkv / L.HG;
    // Chunks are sized by estimated time: a token's bytes (a dense FP32 token
    // moves ~10x the bytes of a packed one), packed bytes weighted 1.4x for
    // their lower streaming rate.  About eight CTAs of work per SM (four waves
    // at two resident CTAs): the block scheduler then balances dense against
    // packed chunks and the last partial wave is short (config 2: 6 / 8 / 12 /
    // 16 CTAs of work per SM measured 598 / 544 / 585 / 588 us per step).  Small launches (a
    // sequence-sharded rank's share) keep at least 512 KB per CTA, while they
    // still fill two waves: per-CTA fixed costs stay small against the streaming.
    const double dense_tok = (double)L.HG * hd * 8.0;
    const double pbs_tok = 1.4 * ((double)L.HG * (hd / 2.0 + 2.0 * hd * 4 / 16.0 + 8.0) + 8.0);
    const double total = (double)L.njobs * L.nhg * (dense_cap * dense_tok + pbs_tok_cap * pbs_tok);
    const double per_cta = std::max({total / (8.0 * 148.0), std::min(524288.0, total / (4.0 * 148.0)), 1.0});
    auto tokens = [](double t, long long lo, long long hi) {
        long long c = ((long long)t + 31) / 32 * 32;
        return (int)std::max(lo, std::min(hi, c));
    };
    L.DC = tokens(per_cta / dense_tok, 32, 1024);
    L.PC = tokens(per_cta / pbs_tok, 64, 4096);
    L.nd = ceil_div(dense_cap, L.DC);
    L.np = ceil_div(pbs_tok_cap, L.PC);
    return TT_OK;
}

// Sets a kernel's dynamic shared-memory limit once per device (a per-device
// function attribute), also when several host threads launch at once; one
// flag set per kernel instantiation.
template <auto Kernel>
static tt_status smem_limit_once(size_t bytes, const char* what) {
    static std::once_flag once[64];
    static cudaError_t err[64];
    int dev = 0;
    cudaGetDevice(&dev);
    std::call_once(once[dev & 63], [&] {
        err[dev & 63] = cudaFuncSetAttribute(Kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
    });
    return err[dev & 63] == cudaSuccess ? TT_OK : check_cuda(err[dev & 63], what);
}

template <int HD, int GM, bool MMA>
static tt_status launch_packed_t(const AttnLaunch& L, cudaStream_t st) {
    size_t mx = 0;
    for (int hg = 1; hg <= 8; ++hg) mx = std::max(mx, kernel_smem_bytes<HD, GM, MMA>(hg, 4));
    tt_status s = smem_limit_once<k_attn_packed<HD, GM, MMA>>(mx, "cudaFuncSetAttribute(k_attn_packed)");
    if (s != TT_OK) return s;
    k_attn_packed<HD, GM, MMA><<<dim3(L.np, L.njobs * L.nhg), NT, kernel_smem_bytes<HD, GM, MMA>(L.HG, L.meta_bytes), st>>>(L);
    return check_launch("k_attn_packed");
}

template <int HD, int GM>
static tt_status launch_dense_t(const AttnLaunch& L, cudaStream_t st) {
    size_t mx = 0;
    for (int hg = 1; hg <= 8; ++hg) mx = std::max(mx, dense_smem_bytes<HD, GM>(hg));
    tt_status s = smem_limit_once<k_attn_dense<HD, GM>>(mx, "cudaFuncSetAttribute(k_attn_dense)");
    if (s != TT_OK) return s;
    k_attn_dense<HD, GM><<<dim3(L.nd, L.njobs * L.nhg), NT, dense_smem_bytes<HD, GM>(L.HG), st>>>(L);
    return check_launch("k_attn_dense");
}

// Packed chunks run on the tensor cores (mma.sync f16) for head_dim 64 / 128,
// up to 4 query heads per kv head (5 to 8 when the kv heads come in groups of
// 4: two warps per kv head), an even number of kv heads and fp16 metadata in
// every job of the batch; other shapes keep the SIMT unit.
template <int HD, int GM>
static tt_status launch_packed_g(const AttnLaunch& L, cudaStream_t st) {
    if constexpr ((HD == 64 || HD == 128) && (GM <= 4 || GM == 8)) {
        if (L.meta_bytes == 2 && (L.HG * L.nhg) % 2 == 0 && (GM <= 4 || L.HG == 4))
            return launch_packed_t<HD, GM, true>(L, st);
    }
    return launch_packed_t<HD, GM, false>(L, st);
}

// which: 0 dense kernel, 1 packed kernel
template <int HD>
static tt_status launch_kind_hd(const AttnLaunch& L, int which, cudaStream_t st) {
    switch (pick_gm(L.G)) {
        case 1: return which ? launch_packed_g<HD, 1>(L, st) : launch_dense_t<HD, 1>(L, st);
        case 2: return which ? launch_packed_g<HD, 2>(L, st) : launch_dense_t<HD, 2>(L, st);
        case 4: return which ? launch_packed_g<HD, 4>(L, st) : launch_dense_t<HD, 4>(L, st);
        case 8:
            if constexpr (HD <= 128) return which ? launch_packed_g<HD, 8>(L, st) : launch_dense_t<HD, 8>(L, st);
            return set_error(TT_ERR_UNSUPPORTED, "head_dim 256 supports at most 4 query heads per kv head");
    }
    return set_error(TT_ERR_UNSUPPORTED, "unsupported GQA ratio");
}

static tt_status launch_kind(const AttnLaunch& L, int which, cudaStream_t st) {
    switch (L.inline_job.hd) {  // callers always fill inline_job.hd/nq (also for engine batches)
        case 16: return launch_kind_hd<16>(L, which, st);
        case 32: return launch_kind_hd<32>(L, which, st);
        case 64: return launch_kind_hd<64>(L, which, st);
        case 128: return launch_kind_hd<128>(L, which, st);
        case 256: return launch_kind_hd<256>(L, which, st);
        default: return set_error(TT_ERR_UNSUPPORTED, "unsupported head_dim");
    }
}

// A second stream per device for the dense kernel, forked from and joined
// back into the caller's stream with events, so that the dense (memory-bound)
// and packed (issue-bound) chunks share the GPU.  Stream capture follows the
// fork into the side stream and back.
struct SideStream {
    std::once_flag once;
    std::mutex mu;
    cudaError_t err = cudaSuccess;
    cudaStream_t s = nullptr;
    cudaEvent_t fork = nullptr, join = nullptr;
};
static SideStream g_side[64];

static tt_status launch_partial_any(const AttnLaunch& L, cudaStream_t st) {
    if (L.nd + L.np == 0) return TT_OK;
    const int ps = prof_begin(1, st);  // the attention phase: both kernels, fork to join
    tt_status s = TT_OK;
    if (L.nd > 0 && L.np > 0) {
        int dev = 0;
        cudaGetDevice(&dev);
        SideStream& S = g_side[dev & 63];
        std::call_once(S.once, [&] {
            S.err = cudaStreamCreateWithFlags(&S.s, cudaStreamNonBlocking);
            if (S.err == cudaSuccess) S.err = cudaEventCreateWithFlags(&S.fork, cudaEventDisableTiming);
            if (S.err == cudaSuccess) S.err = cudaEventCreateWithFlags(&S.join, cudaEventDisableTiming);
        });
        if (S.err != cudaSuccess) return check_cuda(S.err, "side stream");
        std::lock_guard<std::mutex> g(S.mu);
        if ((s = check_cuda(cudaEventRecord(S.fork, st), "fork")) != TT_OK) return s;
        if ((s = check_cuda(cudaStreamWaitEvent(S.s, S.fork, 0), "fork")) != TT_OK) return s;
        s = launch_kind(L, 0, S.s);
        if (s == TT_OK) s = launch_kind(L, 1, st);
        tt_status s2 = check_cuda(cudaEventRecord(S.join, S.s), "join");
        if (s2 == TT_OK) s2 = check_cuda(cudaStreamWaitEvent(st, S.join, 0), "join");
        if (s == TT_OK) s = s2;
    } else {
        s = launch_kind(L, L.nd > 0 ? 0 : 1, st);
    }
    prof_end(ps, st);
    return s;
}

// The partial kernel merges a job's chunks in its last CTA when the caller
// allows it and a job has few chunk slots (the merging CTA walks them alone;
// wide single-job launches keep the nq-CTA merge kernel).
constexpr int kTailMergeMaxChunks = 128;
constexpr int kMergeGroup = 64;  // chunk slots per CTA of the separate head merge
static bool tail_merge(const AttnLaunch& L) {
    return L.merge_mode != 0 && L.nd + L.np > 0 && L.nd + L.np <= kTailMergeMaxChunks;
}

tt_status launch_sharded_partial(const AttnLaunch& L, float* xch, cudaStream_t st) {
    if (tail_merge(L)) {
        AttnLaunch Lm = L;
        Lm.merge_mode = 2;
        Lm.xch = xch;
        return launch_partial_any(Lm, st);
    }
    AttnLaunch L0 = L;
    L0.merge_mode = 0;
    tt_status s = launch_partial_any(L0, st);
    if (s != TT_OK) return s;
    dim3 grid(L.inline_job.nq, L.njobs);
    const int ps = prof_begin(2, st);  // the sharded epilogue kernels count as finalize
    // peer exchange: the rows go to this rank's slot of its own region first
    float* dst = L.px.world > 1
                     ? L.px.rows[L.px.rank] + (size_t)L.px.rank * L.px.jobs * L.inline_job.nq * (L.inline_job.hd + 2)
                     : xch;
    k_shard_local_merge<<<grid, NT, (size_t)(L.nd + L.np + 1) * sizeof(float), st>>>(L, dst);
    tt_status s2 = check_launch("k_shard_local_merge");
    if (s2 == TT_OK && L.px.world > 1) {
        k_publish_rows<<<L.njobs, NT, 0, st>>>(L);
        s2 = check_launch("k_publish_rows");
    }
    prof_end(ps, st);
    return s2;
}

tt_status launch_sharded_merge(const AttnLaunch& L, const float* xch_all, RouteRow* route, int pos_cap,
                               cudaStream_t st) {
    // enough CTAs for the job's outputs (nq x hd values, about four per thread)
    // and for its positions (four per thread), at most one wave (3 CTAs per SM)
    // over the launch: a CTA's fixed cost (descriptor, counters, the heads'
    // (M, L)) is a chain of dependent loads, so fewer, fuller CTAs finish sooner
    // (config 5, one rank of 8: 38.8 -> 35.6 us; of 1: 113 -> 100 us)
    const int outs = ceil_div(L.inline_job.nq * L.inline_job.hd, 4 * NT);
    const int gx = std::max(1, std::min(std::max(outs, ceil_div(std::max(pos_cap, 1), 4 * NT)),
                                        std::max(1, 3 * 148 / L.njobs)));
    dim3 grid(gx, L.njobs);
    const int ps = prof_begin(2, st);
    k_shard_merge<<<grid, NT, (size_t)2 * L.inline_job.nq * sizeof(float), st>>>(L, xch_all, route);
    prof_end(ps, st);
    return check_launch("k_shard_merge");
}

// L.inline_job.hd / .nq must be set for engine batches too (they select the
// kernel instantiation and the merge shared memory).
tt_status launch_attention(const AttnLaunch& L, cudaStream_t st) {
    const bool fused = tail_merge(L);
    {
        AttnLaunch Lp = L;
        Lp.merge_mode = fused ? 1 : 0;
        tt_status s = launch_partial_any(Lp, st);
        if (s != TT_OK) return s;
    }
    const int nq = L.inline_job.nq;
    if (!fused) {
        // up to kMergeGroup chunk slots per job in one pass, else two
        const int nch = L.nd + L.np;
        const int groups = ceil_div(nch, kMergeGroup);
        const size_t sm = ((size_t)std::max(kMergeGroup, groups) + 1 + (size_t)NW * L.inline_job.hd) * sizeof(float);
        const int ps = prof_begin(2, st);
        if (groups > 1) {
            k_attn_merge_heads<<<dim3(nq, L.njobs, groups), NT, sm, st>>>(L, kMergeGroup, 1, 0);
            tt_status s = check_launch("k_attn_merge_heads");
            if (s != TT_OK) return s;
        }
        k_attn_merge_heads<<<dim3(nq, L.njobs, 1), NT, sm, st>>>(L, groups > 1 ? groups : nch,
                                                                   groups > 1 ? kMergeGroup : 1, 1);
        prof_end(ps, st);
        tt_status s = check_launch("k_attn_merge_heads");
        if (s != TT_OK) return s;
    }
    // positions: at most nd * DC dense + np * PC packed; one wave over the
    // launch (4 CTAs per SM), each CTA striding over its job's positions four
    // per thread (measured on config 2: 38.4 -> 36.3 us against two waves)
    const long long tcap = (long long)L.nd * L.DC + (long long)L.np * L.PC;
    const long long gx = std::min<long long>((tcap + 4 * NT - 1) / (4 * NT), std::max(1, 4 * 148 / L.njobs));
    dim3 grid((unsigned)std::max<long long>(1, gx), L.njobs);
    const int ps = prof_begin(2, st);
    k_attn_weights<<<grid, NT, (size_t)2 * nq * sizeof(float), st>>>(L);
    prof_end(ps, st);
    return check_launch("k_attn_weights");
}

// ---------------------------------------------------------------------------
// stand-alone entry point with a per-device workspace
// ---------------------------------------------------------------------------
struct Workspace {
    float* buf = nullptr;
    size_t floats = 0;
};
static Workspace g_ws[64];

static tt_status workspace(int dev, size_t floats, float** out) {
    Workspace& w = g_ws[dev & 63];
    if (w.floats < floats) {
        if (w.buf) cudaFree(w.buf);
        w.buf = nullptr;
        w.floats = 0;
        size_t n = std::max(floats, (size_t)1 << 20);
        tt_status s = check_cuda(cudaMalloc(&w.buf, n * sizeof(float)), "cudaMalloc(attention workspace)");
        if (s != TT_OK) return s;
        w.floats = n;
    }
    *out = w.buf;
    return TT_OK;
}

static bool aligned16(const void* p) { return ((uintptr_t)p & 15) == 0; }

}  // namespace tt

using namespace tt;

extern "C" tt_status tt_device_error(int clear, int* out) {
    if (!out) return set_error(TT_ERR_INVALID_ARGUMENT, "NULL argument.");
    tt_status s = check_cuda(cudaDeviceSynchronize(), "tt_device_error");
    if (s != TT_OK) return s;
    s = check_cuda(cudaMemcpyFromSymbol(out, g_device_error, sizeof(int)), "tt_device_error");
    if (s != TT_OK) return s;
    if (clear) {
        const int zero = 0;
        s = check_cuda(cudaMemcpyToSymbol(g_device_error, &zero, sizeof(int)), "tt_device_error");
    }
    return s;
}

extern "C" tt_status tt_fused_attention_decode(const float* Q, const float* dense_K, const float* dense_V,
                                               int dense_count, const int32_t* PBS_K_Packed,
                                               const void* PBS_K_Scales, const void* PBS_K_Zeroes,
                                               const int32_t* PBS_V_Packed, const void* PBS_V_Scales,
                                               const void* PBS_V_Zeroes, const int64_t* PBS_token_ids,
                                               int num_blocks, int num_q_heads, int num_kv_heads, int head_dim,
                                               float* attn_output, float* mean_attn_weights, int k_group_size,
                                               int meta_fp16, void* stream) {
    if (dense_count < 0) return set_error(TT_ERR_INVALID_ARGUMENT, "dense_count must be non-negative.");
    if (num_blocks < 0) return set_error(TT_ERR_INVALID_ARGUMENT, "num_blocks must be non-negative.");
    if (num_q_heads <= 0 || num_kv_heads <= 0 || head_dim <= 0)
        return set_error(TT_ERR_INVALID_ARGUMENT, "num_q_heads, num_kv_heads, and head_dim must be positive integers.");
    if (k_group_size != 16 && k_group_size != 32)
        return set_error(TT_ERR_INVALID_ARGUMENT, "k_group_size must be 16 or 32.");
    if (!Q || !attn_output) return set_error(TT_ERR_INVALID_ARGUMENT, "Q and attn_output must not be NULL.");
    if (dense_count > 0 && (!dense_K || !dense_V))
        return set_error(TT_ERR_INVALID_ARGUMENT, "dense_K/dense_V must not be NULL when dense_count > 0.");
    if (num_blocks > 0 && (!PBS_K_Packed || !PBS_K_Scales || !PBS_K_Zeroes || !PBS_V_Packed || !PBS_V_Scales ||
                           !PBS_V_Zeroes || !PBS_token_ids))
        return set_error(TT_ERR_INVALID_ARGUMENT, "PBS pointers must not be NULL when num_blocks > 0.");
    if (num_blocks > 0 && head_dim % 16 != 0)
        return set_error(TT_ERR_UNSUPPORTED, "head_dim must be a multiple of 16 for packed V rows.");
    if (!aligned16(Q) || (dense_count > 0 && (!aligned16(dense_K) || !aligned16(dense_V))) ||
        (num_blocks > 0 && (!aligned16(PBS_K_Packed) || !aligned16(PBS_V_Packed) || !aligned16(PBS_K_Scales) ||
                            !aligned16(PBS_K_Zeroes) || !aligned16(PBS_V_Scales) || !aligned16(PBS_V_Zeroes) ||
                            !aligned16(PBS_token_ids))))
        return set_error(TT_ERR_INVALID_ARGUMENT, "Q, dense_K, dense_V and the PBS buffers must be 16-byte aligned.");

    AttnLaunch L;
    memset(&L, 0, sizeof(L));
    L.njobs = 1;
    const long long ntok_ll = (long long)num_blocks * k_group_size;
    if (ntok_ll + dense_count > INT_MAX)
        return set_error(TT_ERR_INVALID_ARGUMENT, "num_blocks * k_group_size + dense_count exceeds INT_MAX.");
    const int ntok = (int)ntok_ll;
    tt_status s = plan_attention(L, num_q_heads, num_kv_heads, head_dim, dense_count, ntok);
    if (s != TT_OK) return s;
    int dev = 0;
    s = check_cuda(cudaGetDevice(&dev), "cudaGetDevice");
    if (s != TT_OK) return s;
    const int T = dense_count + ntok;
    const int maxch = L.nd + L.np;
    const size_t stride = ((size_t)std::max(T, 1) + 3) / 4 * 4;  // float4 logit rows
    const size_t ml_floats = ((size_t)maxch * num_q_heads * 2 + 3) / 4 * 4;
    const size_t need = ml_floats + (size_t)maxch * num_q_heads * head_dim + (size_t)num_q_heads * stride + 64;
    float* ws = nullptr;
    s = workspace(dev, need, &ws);
    if (s != TT_OK) return s;

    JobDesc& J = L.inline_job;
    J.nq = num_q_heads; J.nkv = num_kv_heads; J.hd = head_dim; J.grp = k_group_size; J.meta16 = meta_fp16 ? 1 : 0;
    J.n0 = dense_count; J.n1 = 0; J.n2 = 0; J.ring_head = 0; J.ring_size = 0; J.nblk = num_blocks;
    J.K0 = dense_K; J.V0 = dense_V; J.K1 = J.V1 = J.K2 = J.V2 = nullptr;
    J.kp = PBS_K_Packed; J.ks = PBS_K_Scales; J.kz = PBS_K_Zeroes;
    J.vp = PBS_V_Packed; J.vs = PBS_V_Scales; J.vz = PBS_V_Zeroes; J.ids = PBS_token_ids;
    J.ctr = nullptr;
    J.part_ml = ws;
    J.part_acc = ws + ml_floats;
    J.scores = J.part_acc + (size_t)maxch * num_q_heads * head_dim;
    J.score_stride = (int)stride;
    J.max_chunks = maxch;
    J.g = nullptr; J.hh_scores = nullptr; J.hh_ids = nullptr; J.decay = 0.f; J.msl = 0;
    L.jobs[0] = nullptr;
    L.meta_bytes = meta_fp16 ? 2 : 4;
    L.Q[0] = Q;
    L.out[0] = attn_output;
    L.mw[0] = mean_attn_weights;
    return launch_attention(L, (cudaStream_t)stream);
}
