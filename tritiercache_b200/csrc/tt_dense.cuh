// tt_dense.cuh -- k_attn_dense: split-KV decode attention over the FP32 dense
// tiers (sinks, heavy hitters, recent ring) of one chunk of positions for one
// kv-head group.  Included by tt_attn.cu after tt_partial.cuh.
//
// The dense tiers are a pure stream (1 KB of K+V per token and kv head at
// head_dim 128, about 1 FLOP per byte), so this kernel is built for memory
// parallelism: per stage of NTOK positions one lane of warp 0 per position
// issues two 1-D TMA bulk copies (its K and V rows of the group's HG kv heads,
// one contiguous span of the token's row each) into shared memory, completion
// counted on the stage's mbarrier; NS stages are in flight, and the rows of
// the stage NS further on are prefetched into L2 (cp.async.bulk.prefetch) as
// each stage is issued, so about 2 NS stages of bytes are outstanding without
// more shared memory.  Every mbarrier wait is bounded (TT_ERR_TIMEOUT recorded
// on expiry, own copies drained).  No register holds data in flight.
//
// Per stage each warp takes TPW positions of its kv head (warp % HG):
//   QK   lane <-> channels (consecutive 16-byte shared-memory reads, no bank
//        conflicts), TPW x GM partial dots reduced with one reduce-scatter
//        butterfly; the logits go through a small per-warp table so that
//        every lane holds all TPW x GM of them;
//   online softmax in log2 units, replicated in every lane (no broadcast);
//   PV   lane <-> channels, f32x2 FMAs.
// The warps sharing a kv head merge their (m, l, acc) at the end of the chunk.
#pragma once

namespace tt {

constexpr int kDenseNS = 3;    // stages in flight (shared memory)
constexpr int kDenseTPW = 4;   // positions per warp per stage

// Positions per stage: TPW for every warp of the group's heads.
__host__ __device__ __forceinline__ int dense_stage_tokens(int HG) { return kDenseTPW * (NW / HG); }
// One stage: [NTOK][HG][HD] floats of K, then the same of V.
__host__ __device__ __forceinline__ int dense_stage_bytes(int HD, int HG) {
    return 2 * dense_stage_tokens(HG) * HG * HD * 4;
}
template <int HD, int GM>
__host__ __device__ __forceinline__ size_t dense_smem_bytes(int HG) {
    const size_t stages = (size_t)kDenseNS * dense_stage_bytes(HD, HG);
    const size_t merge = (size_t)NW * GM * (HD + 2) * 4;
    const size_t tabs = (size_t)NW * kDenseTPW * GM * 4;  // per-warp logit tables
    return (stages > merge ? stages : merge) + tabs;
}

__device__ __forceinline__ void prefetch_l2(const void* src, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}

// Issues the bulk copies of stage s (positions [t0 + s*NTOK, ...) of [t0, t1))
// and the L2 prefetch of stage s + NS.  Every copy starts 16-byte aligned (row
// offsets are multiples of HD*4 bytes and the tier bases are 16-byte aligned)
// and moves HG*HD*4 bytes.
template <int HD>
__device__ __forceinline__ void dense_issue_stage(const JobDesc& J, const TierCounts& tc, int HG, int h0, int t0,
                                                  int t1, int s, unsigned char* stages, uint64_t* bars, int lane) {
    const int NTOK = dense_stage_tokens(HG);
    const int s0 = t0 + s * NTOK;
    const int nt = min(NTOK, t1 - s0);
    const uint32_t row = (uint32_t)HG * HD * 4;
    unsigned char* buf = stages + (size_t)(s % kDenseNS) * dense_stage_bytes(HD, HG);
    uint64_t* bar = &bars[s % kDenseNS];
    if (lane == 0) mbar_expect_tx(bar, 2u * nt * row);
    __syncwarp();
    if (lane < nt) {
        const float *Kb, *Vb;
        int slot;
        dense_slot(J, tc, s0 + lane, Kb, Vb, slot);
        const size_t off = (size_t)slot * J.nkv * HD + (size_t)h0 * HD;
        tma_load_1d(buf + (size_t)lane * row, Kb + off, row, bar);
        tma_load_1d(buf + (size_t)(NTOK + lane) * row, Vb + off, row, bar);
    }
    const int p0 = s0 + kDenseNS * NTOK;  // the stage NS further on
    if (lane < min(NTOK, t1 - p0)) {
        const float *Kb, *Vb;
        int slot;
        dense_slot(J, tc, p0 + lane, Kb, Vb, slot);
        const size_t off = (size_t)slot * J.nkv * HD + (size_t)h0 * HD;
        prefetch_l2(Kb + off, row);
        prefetch_l2(Vb + off, row);
    }
}

// grid (nd, njobs * nhg).  With merge_mode set the job's last CTA (of this
// kernel or of the packed one) merges the job's chunks.
template <int HD, int GM>
__global__ void __launch_bounds__(NT, 2) k_attn_dense(const __grid_constant__ AttnLaunch L) {
    constexpr int CPL = HDT<HD>::CPL;  // channels per lane (HD >= 32; HD = 16 uses half the lanes)
    constexpr int NV = kDenseTPW * GM; // logits per warp and stage
    extern __shared__ __align__(128) unsigned char smem[];
    __shared__ __align__(8) uint64_t bars[kDenseNS];
    __shared__ JobDesc Js;
    __shared__ TierCounts Ts;
    const int job = blockIdx.y / L.nhg;
    const int hg = blockIdx.y - job * L.nhg;
    if (threadIdx.x == 0) {
        Js = L.jobs[job] ? *L.jobs[job] : L.inline_job;
        Ts = resolve_counts(Js);
#pragma unroll
        for (int i = 0; i < kDenseNS; ++i) mbar_init(&bars[i], 1);
        mbar_fence_init();
    }
    __syncthreads();
    const JobDesc& J = Js;
    const TierCounts tc = Ts;
    const int D = tc.n0 + tc.n1 + tc.n2;
    const ShardRange R = shard_range(D, tc.nblk, J.grp, L.rank, L.world);
    const int t0 = R.dlo + (int)blockIdx.x * L.DC;
    const int t1 = min(R.dhi, t0 + L.DC);
    const int G = L.G, HG = L.HG;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int kvl = warp % HG, r0 = warp / HG, WPH = NW / HG;
    const bool active = warp < HG * WPH;
    const int kvh = hg * HG + kvl;
    const int NTOK = dense_stage_tokens(HG);
    const int nst = t0 < t1 ? ceil_div(t1 - t0, NTOK) : 0;
    unsigned char* stages = smem;
    float* tab = reinterpret_cast<float*>(smem + (dense_smem_bytes<HD, GM>(HG) - (size_t)NW * NV * 4)) + warp * NV;
    if (warp == 0)
        for (int s = 0; s < kDenseNS && s < nst; ++s)
            dense_issue_stage<HD>(J, tc, HG, hg * HG, t0, t1, s, stages, bars, lane);

    // this lane's query channels for the GM heads of its kv head (zero rows past G)
    const int c0 = lane * CPL;
    const bool lane_on = c0 < HD;
    float q[GM][CPL];
    {
        const float* __restrict__ Qj = L.Q[job];
#pragma unroll
        for (int g = 0; g < GM; ++g)
#pragma unroll
            for (int j = 0; j < CPL; ++j)
                q[g][j] = (active && g < G && lane_on) ? Qj[((size_t)kvh * G + g) * HD + c0 + j] : 0.f;
    }
    const float sc = (1.0f / sqrtf((float)HD)) * kLog2e;
    float m[GM], l[GM], acc[GM][CPL];
#pragma unroll
    for (int g = 0; g < GM; ++g) {
        m[g] = -INFINITY;
        l[g] = 0.f;
#pragma unroll
        for (int j = 0; j < CPL; ++j) acc[g][j] = 0.f;
    }
    const size_t row = (size_t)HG * HD;  // floats per staged position
    bool failed = false;
    int s = 0;
    for (; s < nst; ++s) {
        const bool ok = mbar_wait_bounded(&bars[s % kDenseNS], (uint32_t)((s / kDenseNS) & 1));
        if (__syncthreads_or(!ok)) {
            failed = true;
            break;
        }
        const float* Ks = reinterpret_cast<const float*>(stages + (size_t)(s % kDenseNS) * dense_stage_bytes(HD, HG));
        const float* Vs = Ks + (size_t)NTOK * row;
        const int s0 = t0 + s * NTOK;
        const int nt = min(NTOK, t1 - s0);
        // this warp's positions of the stage: r0, r0 + WPH, ... (TPW of them)
        const int ntw = active ? max(0, min(kDenseTPW, (nt - r0 + WPH - 1) / WPH)) : 0;
        if (ntw > 0) {
            // ---- QK partials: a[t*GM + g] ----
            float a[NV];
#pragma unroll
            for (int t = 0; t < kDenseTPW; ++t) {
                float k[CPL];
                const float* kr = Ks + (size_t)(r0 + t * WPH) * row + (size_t)kvl * HD + c0;
                if (t < ntw && lane_on) {
                    if constexpr (CPL % 4 == 0) {
#pragma unroll
                        for (int j = 0; j < CPL; j += 4) {
                            const float4 x = *reinterpret_cast<const float4*>(kr + j);
                            k[j] = x.x; k[j + 1] = x.y; k[j + 2] = x.z; k[j + 3] = x.w;
                        }
                    } else if constexpr (CPL == 2) {
                        const float2 x = *reinterpret_cast<const float2*>(kr);
                        k[0] = x.x; k[1] = x.y;
                    } else {
                        k[0] = kr[0];
                    }
                } else {
#pragma unroll
                    for (int j = 0; j < CPL; ++j) k[j] = 0.f;
                }
#pragma unroll
                for (int g = 0; g < GM; ++g) {
                    float d = 0.f;
#pragma unroll
                    for (int j = 0; j < CPL; ++j) d = fmaf(q[g][j], k[j], d);
                    a[t * GM + g] = d;
                }
            }
            warp_reduce_scatter_to_smem<NV>(a, tab, lane);
            __syncwarp();
            // ---- every lane: the TPW x GM logits (log2 units) ----
            float sl[kDenseTPW][GM];
#pragma unroll
            for (int t = 0; t < kDenseTPW; ++t) {
#pragma unroll
                for (int g = 0; g < GM; ++g) {
                    const float v = tab[t * GM + g] * sc;
                    sl[t][g] = (t < ntw && g < G) ? v : -INFINITY;
                }
            }
            // logits to scratch for the mean weights: lane i < NV stores value i
            if (lane < NV) {
                const int t = lane / GM, g = lane % GM;
                if (t < ntw && g < G)
                    J.scores[(size_t)(kvh * G + g) * J.score_stride + s0 + r0 + t * WPH] = tab[lane] * sc;
            }
            __syncwarp();  // the table is rewritten next stage
            // ---- online softmax per head ----
#pragma unroll
            for (int g = 0; g < GM; ++g) {
                float mu = sl[0][g];
#pragma unroll
                for (int t = 1; t < kDenseTPW; ++t) mu = fmaxf(mu, sl[t][g]);
                const float mn = fmaxf(m[g], mu);
                float alpha = 1.f, ps = 0.f;
                if (mn != -INFINITY) {
                    alpha = ex2_fast(m[g] - mn);
#pragma unroll
                    for (int t = 0; t < kDenseTPW; ++t) {
                        sl[t][g] = sl[t][g] == -INFINITY ? 0.f : ex2_fast(sl[t][g] - mn);
                        ps += sl[t][g];
                    }
                } else {
#pragma unroll
                    for (int t = 0; t < kDenseTPW; ++t) sl[t][g] = 0.f;
                }
                m[g] = mn;
                l[g] = fmaf(l[g], alpha, ps);
#pragma unroll
                for (int j = 0; j < CPL; ++j) acc[g][j] *= alpha;
            }
            // ---- PV ----
#pragma unroll
            for (int t = 0; t < kDenseTPW; ++t) {
                if (t < ntw && lane_on) {
                    const float* vr = Vs + (size_t)(r0 + t * WPH) * row + (size_t)kvl * HD + c0;
                    float v[CPL];
                    if constexpr (CPL % 4 == 0) {
#pragma unroll
                        for (int j = 0; j < CPL; j += 4) {
                            const float4 x = *reinterpret_cast<const float4*>(vr + j);
                            v[j] = x.x; v[j + 1] = x.y; v[j + 2] = x.z; v[j + 3] = x.w;
                        }
                    } else if constexpr (CPL == 2) {
                        const float2 x = *reinterpret_cast<const float2*>(vr);
                        v[0] = x.x; v[1] = x.y;
                    } else {
                        v[0] = vr[0];
                    }
                    if constexpr (CPL % 2 == 0) {
#pragma unroll
                        for (int g = 0; g < GM; ++g) {
                            const u64 pp = f2pack(sl[t][g], sl[t][g]);
#pragma unroll
                            for (int j = 0; j < CPL; j += 2) {
                                const float2 r = f2unpack(ffma2(pp, f2pack(v[j], v[j + 1]), f2pack(acc[g][j], acc[g][j + 1])));
                                acc[g][j] = r.x;
                                acc[g][j + 1] = r.y;
                            }
                        }
                    } else {
#pragma unroll
                        for (int g = 0; g < GM; ++g) acc[g][0] = fmaf(sl[t][g], v[0], acc[g][0]);
                    }
                }
            }
        }
        __syncthreads();  // every warp is done with this slot
        if (warp == 0 && s + kDenseNS < nst)
            dense_issue_stage<HD>(J, tc, HG, hg * HG, t0, t1, s + kDenseNS, stages, bars, lane);
    }
    if (failed) {
        // drain this CTA's own copies in flight and give up on the chunk (it
        // still arrives below, so the job's arrival count stays consistent)
        for (int k = s; k < nst && k < s + kDenseNS; ++k)
            (void)mbar_wait_bounded(&bars[k % kDenseNS], (uint32_t)((k / kDenseNS) & 1));
        if (threadIdx.x == 0) {
            atomicCAS(&g_device_error, 0, (int)TT_ERR_TIMEOUT);
            if (J.ctr) atomicCAS(const_cast<int*>(&J.ctr->error), 0, (int)TT_ERR_TIMEOUT);
        }
    } else if (t0 < t1) {
        const int chunk = (int)blockIdx.x;  // dense chunks use the first partial slots
        if (WPH == 1) {
            if (active) {
#pragma unroll
                for (int g = 0; g < GM; ++g) {
                    if (g >= G) break;
                    const size_t pi = part_index(J, chunk, kvh, G, g);
                    if (lane == 0) {
                        J.part_ml[pi * 2 + 0] = m[g];
                        J.part_ml[pi * 2 + 1] = l[g];
                    }
#pragma unroll
                    for (int j = 0; j < CPL; ++j)
                        if (lane_on) J.part_acc[pi * HD + c0 + j] = acc[g][j];
                }
            }
        } else {
            // merge the WPH warps that share a kv head (buffer aliases the stages)
            float* mbuf = reinterpret_cast<float*>(smem);
            float* mine = mbuf + (size_t)warp * GM * (HD + 2);
#pragma unroll
            for (int g = 0; g < GM; ++g) {
                if (lane == 0) {
                    mine[g * (HD + 2) + 0] = m[g];
                    mine[g * (HD + 2) + 1] = l[g];
                }
#pragma unroll
                for (int j = 0; j < CPL; ++j)
                    if (lane_on) mine[g * (HD + 2) + 2 + c0 + j] = acc[g][j];
            }
            __syncthreads();
            if (r0 == 0 && active) merge_warps<HD, GM>(J, mbuf, chunk, kvh, kvl, HG, WPH, G, lane);
        }
    }
    if (L.merge_mode) chunk_merge_tail<HD>(L, J, tc, job);
}

}  // namespace tt
