// tt_dense.cuh -- k_attn_dense: split-KV decode attention over the FP32 dense
// tiers (sinks, heavy hitters, recent ring) of one chunk of positions for one
// kv-head group.  Included by tt_attn.cu after tt_partial.cuh.
//
// The dense tiers are a pure stream (1 KB of K+V per token and kv head at
// head_dim 128, about 1 FLOP per byte), so this kernel is built for memory
// parallelism: per stage of NTOK positions one lane of warp 0 per position
// issues two 1-D TMA bulk copies (its K and V rows of the group's HG kv heads,
// one contiguous span of the token's row each) into shared memory, completion
// counted on the stage's mbarrier; two stages are in flight (an L2 prefetch of
// the stages after them measured slower: 5.1 -> 4.4 TB/s).  Every mbarrier wait is bounded (TT_ERR_TIMEOUT recorded
// on expiry, own copies drained).  No register holds data in flight.
//
// Per stage each warp takes TPW positions of its kv head (warp % HG):
//   QK   lane <-> channels (consecutive 16-byte shared-memory reads, no bank
//        conflicts), f32x2 FMAs over channel pairs, the TPW x GM partial dots
//        reduced with one reduce-scatter butterfly that leaves each logit in
//        32 / (TPW GM) lanes;
//   online softmax in log2 units distributed the same way (one exp per lane
//        and head-wise max / sum over the lanes of a head); each head's
//        rescale factor and each weight go through a per-warp table as
//        {w, w} pairs, so the PV FMAs take them without register moves;
//   PV   lane <-> channels, f32x2 FMAs.
// The warps sharing a kv head merge their (m, l, acc) at the end of the chunk.
#pragma once

namespace tt {

constexpr int kDenseNS = 2;    // stages in flight (shared memory; 2 leaves room for the packed
                               // kernel's CTAs when both run at once: config 2 585 -> 562 us, against 3)
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
    const size_t tabs = (size_t)NW * (kDenseTPW + 1) * GM * 8;  // per-warp {w, w} / {alpha, alpha} tables
    return (stages > merge ? stages : merge) + tabs;
}

// Sum of v[0..N) over the warp, scattered: every lane returns the total of
// value (lane >> (5 - log2 N)); 32 / N adjacent lanes hold the same value.
template <int N>
__device__ __forceinline__ float warp_reduce_scatter(float (&v)[N], int lane) {
    static_assert((N & (N - 1)) == 0 && N <= 32, "power of two");
    int cnt = N;
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) {
        if (cnt > 1) {
            const int half = cnt / 2;
            const bool up = (lane & o) != 0;
#pragma unroll
            for (int i = 0; i < N / 2; ++i) {
                if (i < half) {
                    const float send = up ? v[i] : v[i + half];
                    const float keep = up ? v[i + half] : v[i];
                    v[i] = keep + __shfl_xor_sync(0xffffffffu, send, o);
                }
            }
            cnt = half;
        } else {
            v[0] += __shfl_xor_sync(0xffffffffu, v[0], o);
        }
    }
    return v[0];
}

// Issues the bulk copies of stage s (positions [t0 + s*NTOK, ...) of [t0, t1)).
// Every copy starts 16-byte aligned (row
// offsets are multiples of HD*4 bytes and the tier bases are 16-byte aligned)
// and moves HG*HD*4 bytes.
template <int HD>
__device__ __forceinline__ void dense_issue_stage(const JobDesc& J, const TierCounts& tc, int HG, int h0, int t0,
                                                  int t1, int s, unsigned char* stages, uint64_t* bars, int lane,
                                                  int rank, int world) {
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
        dense_slot(J, tc, s0 + lane, rank, world, Kb, Vb, slot);
        const size_t off = (size_t)slot * J.nkv * HD + (size_t)h0 * HD;
        tma_load_1d(buf + (size_t)lane * row, Kb + off, row, bar);
        tma_load_1d(buf + (size_t)(NTOK + lane) * row, Vb + off, row, bar);
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
    const ShardMap M = shard_map(tc, J.grp, L.rank, L.world);
    const int t0 = (int)blockIdx.x * L.DC;  // this rank's local dense positions [t0, t1)
    const int t1 = min(M.nd, t0 + L.DC);
    const int G = L.G, HG = L.HG;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int kvl = warp % HG, r0 = warp / HG, WPH = NW / HG;
    const bool active = warp < HG * WPH;
    const int kvh = hg * HG + kvl;
    const int NTOK = dense_stage_tokens(HG);
    const int nst = t0 < t1 ? ceil_div(t1 - t0, NTOK) : 0;
    unsigned char* stages = smem;
    float* tab = reinterpret_cast<float*>(smem + (dense_smem_bytes<HD, GM>(HG) - (size_t)NW * (kDenseTPW + 1) * GM * 8) +
                                          (size_t)warp * (kDenseTPW + 1) * GM * 8);
    if (warp == 0)
        for (int s = 0; s < kDenseNS && s < nst; ++s)
            dense_issue_stage<HD>(J, tc, HG, hg * HG, t0, t1, s, stages, bars, lane, L.rank, L.world);

    // this lane's query channels for the GM heads of its kv head (zero rows past
    // G), as channel pairs for the f32x2 FMAs
    const int c0 = lane * CPL;
    const bool lane_on = c0 < HD;
    constexpr int NP = CPL >= 2 ? CPL / 2 : 1;  // channel pairs per lane
    u64 q2[GM][NP];
    {
        const float* __restrict__ Qj = L.Q[job];
#pragma unroll
        for (int g = 0; g < GM; ++g) {
            float qv[2 * NP];
#pragma unroll
            for (int j = 0; j < 2 * NP; ++j)
                qv[j] = (active && g < G && lane_on && j < CPL) ? Qj[((size_t)kvh * G + g) * HD + c0 + j] : 0.f;
#pragma unroll
            for (int p = 0; p < NP; ++p) q2[g][p] = f2pack(qv[2 * p], qv[2 * p + 1]);
        }
    }
    const float sc = (1.0f / sqrtf((float)HD)) * kLog2e;
    // this lane's logit of each stage: value v = t * GM + g, held by 32 / NV lanes
    constexpr int LOG_NV = NV >= 32 ? 5 : NV >= 16 ? 4 : NV >= 8 ? 3 : NV >= 4 ? 2 : NV >= 2 ? 1 : 0;
    constexpr int SH = 5 - LOG_NV;
    constexpr int LOG_GM = GM >= 8 ? 3 : GM >= 4 ? 2 : GM >= 2 ? 1 : 0;
    const int my_v = lane >> SH, my_g = my_v & (GM - 1), my_t = my_v >> LOG_GM;
    const bool my_first = (lane & ((1 << SH) - 1)) == 0;
    float m_h = -INFINITY, l_h = 0.f;  // running max / sum of head my_g
    u64 acc2[GM][NP];
#pragma unroll
    for (int g = 0; g < GM; ++g)
#pragma unroll
        for (int p = 0; p < NP; ++p) acc2[g][p] = 0ull;
    u64* wtab = reinterpret_cast<u64*>(tab);  // [TPW][GM] {w, w}, then [GM] {alpha, alpha}
    u64* atab = wtab + kDenseTPW * GM;
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
                u64 k2[NP];
                const float* kr = Ks + (size_t)(r0 + t * WPH) * row + (size_t)kvl * HD + c0;
                if (t < ntw && lane_on) {
                    if constexpr (CPL % 4 == 0) {
#pragma unroll
                        for (int j = 0; j < CPL; j += 4) {
                            const ulonglong2 x = *reinterpret_cast<const ulonglong2*>(kr + j);
                            k2[j / 2] = x.x;
                            k2[j / 2 + 1] = x.y;
                        }
                    } else if constexpr (CPL == 2) {
                        k2[0] = *reinterpret_cast<const u64*>(kr);
                    } else {
                        k2[0] = f2pack(kr[0], 0.f);
                    }
                } else {
#pragma unroll
                    for (int p = 0; p < NP; ++p) k2[p] = 0ull;
                }
#pragma unroll
                for (int g = 0; g < GM; ++g) {
                    u64 d = fmul2(q2[g][0], k2[0]);
#pragma unroll
                    for (int p = 1; p < NP; ++p) d = ffma2(q2[g][p], k2[p], d);
                    const float2 dd = f2unpack(d);
                    a[t * GM + g] = dd.x + dd.y;
                }
            }
            // ---- the lane's logit (log2 units), its head's online softmax ----
            float sv = warp_reduce_scatter<NV>(a, lane) * sc;
            if (my_t >= ntw || my_g >= G) sv = -INFINITY;
            if (my_first && sv != -INFINITY)
                st_logit(J.scores + (size_t)(kvh * G + my_g) * J.score_stride + s0 + r0 + my_t * WPH, sv);
            float mu = sv;
#pragma unroll
            for (int o = 1 << (SH + LOG_GM); o < 32; o <<= 1) mu = fmaxf(mu, __shfl_xor_sync(0xffffffffu, mu, o));
            const float mn = fmaxf(m_h, mu);
            const float alpha = mn == -INFINITY ? 1.f : ex2_fast(m_h - mn);
            const float pw = sv == -INFINITY ? 0.f : ex2_fast(sv - mn);
            float ps = pw;
#pragma unroll
            for (int o = 1 << (SH + LOG_GM); o < 32; o <<= 1) ps += __shfl_xor_sync(0xffffffffu, ps, o);
            l_h = fmaf(l_h, alpha, ps);
            m_h = mn;
            if (my_first) {
                wtab[my_v] = f2pack(pw, pw);
                if (my_t == 0) atab[my_g] = f2pack(alpha, alpha);
            }
            __syncwarp();
            // ---- rescale and PV ----
#pragma unroll
            for (int g = 0; g < GM; ++g) {
                const u64 al = atab[g];
#pragma unroll
                for (int p = 0; p < NP; ++p) acc2[g][p] = fmul2(acc2[g][p], al);
            }
#pragma unroll
            for (int t = 0; t < kDenseTPW; ++t) {
                if (t < ntw && lane_on) {
                    const float* vr = Vs + (size_t)(r0 + t * WPH) * row + (size_t)kvl * HD + c0;
                    u64 v2[NP];
                    if constexpr (CPL % 4 == 0) {
#pragma unroll
                        for (int j = 0; j < CPL; j += 4) {
                            const ulonglong2 x = *reinterpret_cast<const ulonglong2*>(vr + j);
                            v2[j / 2] = x.x;
                            v2[j / 2 + 1] = x.y;
                        }
                    } else if constexpr (CPL == 2) {
                        v2[0] = *reinterpret_cast<const u64*>(vr);
                    } else {
                        v2[0] = f2pack(vr[0], 0.f);
                    }
                    u64 w[GM];
                    if constexpr (GM % 2 == 0) {
#pragma unroll
                        for (int g = 0; g < GM; g += 2) {
                            const ulonglong2 x = reinterpret_cast<const ulonglong2*>(wtab + t * GM)[g / 2];
                            w[g] = x.x;
                            w[g + 1] = x.y;
                        }
                    } else {
                        w[0] = wtab[t * GM];
                    }
#pragma unroll
                    for (int g = 0; g < GM; ++g)
#pragma unroll
                        for (int p = 0; p < NP; ++p) acc2[g][p] = ffma2(w[g], v2[p], acc2[g][p]);
                }
            }
        }
        __syncthreads();  // every warp is done with this slot
        if (warp == 0 && s + kDenseNS < nst)
            dense_issue_stage<HD>(J, tc, HG, hg * HG, t0, t1, s + kDenseNS, stages, bars, lane, L.rank, L.world);
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
        float mg[GM], lg[GM], og[GM][2 * NP];
#pragma unroll
        for (int g = 0; g < GM; ++g) {
            mg[g] = __shfl_sync(0xffffffffu, m_h, g << SH);  // lane of value (t = 0, g)
            lg[g] = __shfl_sync(0xffffffffu, l_h, g << SH);
#pragma unroll
            for (int p = 0; p < NP; ++p) {
                const float2 x = f2unpack(acc2[g][p]);
                og[g][2 * p] = x.x;
                og[g][2 * p + 1] = x.y;
            }
        }
        if (WPH == 1) {
            if (active) {
#pragma unroll
                for (int g = 0; g < GM; ++g) {
                    if (g >= G) break;
                    const size_t pi = part_index(J, chunk, kvh, G, g);
                    if (lane == 0) {
                        J.part_ml[pi * 2 + 0] = mg[g];
                        J.part_ml[pi * 2 + 1] = lg[g];
                    }
#pragma unroll
                    for (int j = 0; j < CPL; ++j)
                        if (lane_on) J.part_acc[pi * HD + c0 + j] = og[g][j];
                }
            }
        } else {
            // merge the WPH warps that share a kv head (buffer aliases the stages)
            float* mbuf = reinterpret_cast<float*>(smem);
            float* mine = mbuf + (size_t)warp * GM * (HD + 2);
#pragma unroll
            for (int g = 0; g < GM; ++g) {
                if (lane == 0) {
                    mine[g * (HD + 2) + 0] = mg[g];
                    mine[g * (HD + 2) + 1] = lg[g];
                }
#pragma unroll
                for (int j = 0; j < CPL; ++j)
                    if (lane_on) mine[g * (HD + 2) + 2 + c0 + j] = og[g][j];
            }
            __syncthreads();
            if (r0 == 0 && active) merge_warps<HD, GM>(J, mbuf, chunk, kvh, kvl, HG, WPH, G, lane);
        }
    }
    if (L.merge_mode) chunk_merge_tail<HD>(L, J, tc, job);
}

}  // namespace tt
