// tt_weights.cuh -- head-mean attention weights and the decayed score
// feedback of one position, shared by k_attn_weights (tt_attn.cu) and the
// weights items of the partial kernel (tt_partial.cuh).
#pragma once
#include "tt_attn.cuh"

namespace tt {

__device__ __forceinline__ float ex2_fast(float x) {  // 2^x, PTX ex2.approx (rel. error ~2^-22; -inf -> 0)
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// (M, 1/L) of every head once the job's chunks are merged: the partials'
// last chunk slot (a job's active chunks use at most max_chunks - 2 slots).
__device__ __forceinline__ float* head_ml(const JobDesc& J) {
    return J.part_ml + (size_t)(J.max_chunks - 1) * J.nq * 2;
}

// Smallest (score, heavy-hitter slot) of a sequence-sharded merge launch, as
// the complement of order_key(score) << 32 | slot so that zero means "none"
// and atomicMax finds the minimum.  It lives in the job's head (M, 1/L) slot,
// which sharded steps do not use otherwise; their partial launch zeroes it.
__device__ __forceinline__ unsigned long long* route_min_word(const JobDesc& J) {
    return reinterpret_cast<unsigned long long*>(head_ml(J));
}

// Weight of position pos averaged over heads: (1/nq) sum_h 2^(s_h - M_h) / L_h,
// skipping -inf logits (fused_attn_avx2.cpp:286-300).  The logits come
// through L2: in the partial kernel other CTAs wrote them during the launch.
__device__ __forceinline__ float mean_weight(const JobDesc& J, const float* Ms, const float* IL, int nq, int pos) {
    const float* sc = J.scores;
    const size_t stride = (size_t)J.score_stride;
    float sw = 0.f;
    int h = 0;
    for (; h + 32 <= nq; h += 32) {  // all 32 loads in flight before the first use
        float v[32];
#pragma unroll
        for (int k = 0; k < 32; ++k) v[k] = __ldcg(sc + (size_t)(h + k) * stride + pos);
#pragma unroll
        for (int k = 0; k < 32; ++k)
            if (v[k] != -INFINITY) sw = fmaf(ex2_fast(v[k] - Ms[h + k]), IL[h + k], sw);
    }
    for (; h < nq; ++h) {
        const float v = __ldcg(sc + (size_t)h * stride + pos);
        if (v != -INFINITY) sw = fmaf(ex2_fast(v - Ms[h]), IL[h], sw);
    }
    return sw / (float)nq;
}

// Head-mean weights of the 4 positions p4 .. p4 + 3 (float4 logit loads; the
// rows must be 16-byte aligned: J.scores and the stride a multiple of 4
// floats).  Ms[h] is the head's max with -inf replaced by +inf (then every
// logit of the head gives 2^-inf = 0, as the scalar form's skip of -inf
// logits does), so the terms and their order match mean_weight exactly.
__device__ __forceinline__ float4 mean_weight4(const JobDesc& J, const float* Ms, const float* IL, int nq, int p4) {
    const float* sc = J.scores + p4;
    const size_t stride = (size_t)J.score_stride;
    float4 sw = make_float4(0.f, 0.f, 0.f, 0.f);
    int h = 0;
    for (; h + 8 <= nq; h += 8) {  // 8 rows in flight before the first use
        float4 v[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) v[k] = __ldcg(reinterpret_cast<const float4*>(sc + (size_t)(h + k) * stride));
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            const float m = Ms[h + k], il = IL[h + k];
            sw.x = fmaf(ex2_fast(v[k].x - m), il, sw.x);
            sw.y = fmaf(ex2_fast(v[k].y - m), il, sw.y);
            sw.z = fmaf(ex2_fast(v[k].z - m), il, sw.z);
            sw.w = fmaf(ex2_fast(v[k].w - m), il, sw.w);
        }
    }
    for (; h < nq; ++h) {
        const float4 v = __ldcg(reinterpret_cast<const float4*>(sc + (size_t)h * stride));
        const float m = Ms[h], il = IL[h];
        sw.x = fmaf(ex2_fast(v.x - m), il, sw.x);
        sw.y = fmaf(ex2_fast(v.y - m), il, sw.y);
        sw.z = fmaf(ex2_fast(v.z - m), il, sw.z);
        sw.w = fmaf(ex2_fast(v.w - m), il, sw.w);
    }
    const float inv = (float)nq;
    return make_float4(sw.x / inv, sw.y / inv, sw.z / inv, sw.w / inv);
}

// Token id at position pos (-1 where there is none) and, for heavy hitters,
// the HH slot: sinks, heavy hitters, the recent ring, the packed tier.
__device__ __forceinline__ long long position_id(const JobDesc& J, const TierCounts& tc, int D, int pos, int& hh) {
    hh = -1;
    if (pos < tc.n0) return pos;
    if (pos < tc.n0 + tc.n1) {
        hh = pos - tc.n0;
        return J.hh_ids[hh];
    }
    if (pos < D) return (long long)tc.total - tc.n2 + (pos - tc.n0 - tc.n1);
    return J.ids[pos - D];
}

// Token id at local position i of a sequence-sharded rank's share (its dense
// positions, then its packed tokens; world <= 1: the global position) and,
// for heavy hitters, the HH slot; -1 where there is none.
__device__ __forceinline__ long long local_position_id(const JobDesc& J, const TierCounts& tc, const ShardMap& M,
                                                       int r, int w, int i, int& hh) {
    hh = -1;
    if (i < M.nd) {
        int slot;
        const int tier = dense_local_slot(tc, i, r, w, slot);
        if (tier == 0) return slot;
        if (tier == 1) {
            hh = slot;
            return J.hh_ids[slot];
        }
        return ring_slot_id(tc, slot);
    }
    return J.ids[packed_global(i - M.nd, r, w)];
}

// The mean weight of position pos (written to mw when given) and, for
// engines, g[id] = decay * g[id] + w for the token there (cache_engine.cpp:
// 511-540): sinks, heavy hitters (whose HH_scores copy follows), the recent
// ring and the packed tier; ids outside [0, max_seq_len) are skipped.  The
// token id and its old score are loaded before the logits, so their latency
// overlaps the logit loads.  Positions hold distinct tokens, so no two
// threads of a launch touch one g entry.
__device__ __forceinline__ void weigh_position(const JobDesc& J, const TierCounts& tc, int D, const float* Ms,
                                               const float* IL, float* mw, int pos) {
    int hh = -1;
    const long long id = J.g ? position_id(J, tc, D, pos, hh) : -1;
    const bool fb = id >= 0 && id < J.msl;
    const float g_old = fb ? J.g[id] : 0.f;
    const float w = mean_weight(J, Ms, IL, J.nq, pos);
    if (mw) mw[pos] = w;
    if (fb) {
        const float nv = fmaf(J.decay, g_old, w);
        J.g[id] = nv;
        if (hh >= 0) J.hh_scores[hh] = nv;
    }
}

}  // namespace tt
