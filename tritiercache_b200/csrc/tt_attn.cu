// tt_attn.cu -- fused single-query decode attention over the tiered KV cache.
//
// Replaces the reference's fused_attention_decode_avx2
// (csrc/cpu/fused_attn_avx2.cpp:145-301), which dequantizes the whole packed
// background store (PBS) into scratch, materialises an nq x T score matrix
// and walks it per query head.  Here the work is split-KV:
//
//   k_attn_partial  grid = (token chunks, jobs x kv-head groups), 8 warps.
//     Each warp owns one kv head and walks 32-token units of its chunk:
//       QK  lane <-> token.  Dense rows: FP32 dot with the G query heads of
//           the kv head (GQA: every K byte is read once).  PBS rows: the
//           block's 2-bit words are staged in shared memory and unpacked in
//           registers; with qs = q*scale and F = 4 + code the score is
//           sum(qs*F) - 4*sum(qs) + sum(q*zero) -- no dequantized copy.
//       online softmax in log2 units (exp2), per-lane partial sums.
//       PV  lane <-> channels.  Dense V rows are read coalesced; packed V
//           words are unpacked in registers with the per-token scale folded
//           into the weight (ws = p*scale) and the zero into a running sum.
//     Output: per (chunk, q head) partial (m, l, acc[hd]) and the raw logits
//     (for the mean attention weights).
//   k_attn_finalize grid = (token ranges, jobs).  Log-sum-exp merge of the
//     partials into attn_output, the head-mean softmax weights
//     (fused_attn_avx2.cpp:286-300) and, for engine jobs, the decayed score
//     feedback g[id] = decay*g[id] + w (cache_engine.cpp:511-540).
#include <algorithm>

#include "tt_attn.cuh"

namespace tt {

constexpr int NT = 256;
constexpr int NW = NT / TT_WARP;
constexpr float kLog2e = 1.4426950408889634f;

template <int HD>
struct HDT {
    static constexpr int CPL = HD >= 32 ? HD / 32 : 1;  // channels per lane in PV
    static constexpr int DQ = HD / 16;                  // packed V words per (token, head)
};

// 4 + code as a float, code = the 2-bit field of `w` at bit `bit` (rot = (21 - bit) & 31):
// rotate the field to mantissa bits 21-22 and set the exponent of [4, 8).
__device__ __forceinline__ float unpack_4pc(uint32_t w, int rot) {
    return __uint_as_float((__funnelshift_l(w, w, rot) & 0x00600000u) | 0x40800000u);
}

struct WarpSmem {
    uint32_t* kw;      // [2][HD]
    float* qs;         // [2][HD][GM]
    uint32_t* vw;      // [32][DQ]
    float* ws;         // [32][GM]
    const float** vrow;  // [32]
};

template <int HD, int GM>
struct SmemPlan {
    static constexpr int kw = 2 * HD * 4;
    static constexpr int qs = 2 * HD * GM * 4;
    static constexpr int vw = 32 * (HD / 16) * 4;
    static constexpr int ws = 32 * GM * 4;
    static constexpr int vrow = 32 * 8;
    static constexpr int per_warp = kw + qs + vw + ws + vrow;
    static constexpr int merge = NW * GM * (HD + 2) * 4;
    static size_t bytes(int HG) {
        size_t q = (size_t)HG * GM * HD * 4;
        size_t body = (size_t)NW * per_warp;
        if ((size_t)merge > body) body = merge;
        return q + body;
    }
};

__device__ __forceinline__ void dense_slot(const JobDesc& J, const TierCounts& tc, int i, const float*& Kb,
                                           const float*& Vb, int& slot) {
    if (i < tc.n0) {
        Kb = J.K0; Vb = J.V0; slot = i;
    } else if (i < tc.n0 + tc.n1) {
        Kb = J.K1; Vb = J.V1; slot = i - tc.n0;
    } else {
        Kb = J.K2; Vb = J.V2;
        const int r = i - tc.n0 - tc.n1;
        slot = tc.ring_size > 0 ? (tc.ring_head + r) % tc.ring_size : r;
    }
}

template <int HD, int GM>
__global__ void __launch_bounds__(NT) k_attn_partial(const __grid_constant__ AttnLaunch L) {
    using T = HDT<HD>;
    using SP = SmemPlan<HD, GM>;
    extern __shared__ __align__(16) unsigned char smem[];
    __shared__ JobDesc Js;
    __shared__ TierCounts Ts;

    const int job = blockIdx.y / L.nhg;
    const int hg = blockIdx.y - job * L.nhg;
    if (threadIdx.x == 0) {
        Js = L.jobs[job] ? *L.jobs[job] : L.inline_job;
        Ts = resolve_counts(Js);
    }
    __syncthreads();
    const JobDesc& J = Js;
    const TierCounts tc = Ts;
    const int D = tc.n0 + tc.n1 + tc.n2;
    const int ntok = tc.nblk * J.grp;
    const bool is_dense = (int)blockIdx.x < L.nd;
    int t0, t1;
    if (is_dense) {
        t0 = blockIdx.x * L.DC;
        t1 = min(D, t0 + L.DC);
    } else {
        t0 = (blockIdx.x - L.nd) * L.PC;
        t1 = min(ntok, t0 + L.PC);
    }
    if (t0 >= t1) return;

    const int nq = J.nq, nkv = J.nkv, G = L.G, HG = L.HG;
    const size_t kvs = (size_t)nkv * HD;
    const float* __restrict__ Q = L.Q[job];

    // ---- stage the query rows of this kv-head group: q_s[kvl][g][c] ----
    float* q_s = reinterpret_cast<float*>(smem);
    for (int i = threadIdx.x; i < HG * GM * HD; i += NT) {
        const int c = i % HD, kg = i / HD, g = kg % GM, kvl = kg / GM;
        q_s[i] = g < G ? Q[((size_t)(hg * HG + kvl) * G + g) * HD + c] : 0.f;
    }
    __syncthreads();

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int kvl = warp % HG, r0 = warp / HG, WPH = NW / HG;
    const int kvh = hg * HG + kvl;
    unsigned char* wbase = smem + (size_t)HG * GM * HD * 4 + (size_t)warp * SP::per_warp;
    WarpSmem W;
    W.kw = reinterpret_cast<uint32_t*>(wbase);
    W.qs = reinterpret_cast<float*>(wbase + SP::kw);
    W.vw = reinterpret_cast<uint32_t*>(wbase + SP::kw + SP::qs);
    W.ws = reinterpret_cast<float*>(wbase + SP::kw + SP::qs + SP::vw);
    W.vrow = reinterpret_cast<const float**>(wbase + SP::kw + SP::qs + SP::vw + SP::ws);
    const float* qk = q_s + (size_t)kvl * GM * HD;
    const float sc = (1.0f / sqrtf((float)HD)) * kLog2e;  // log2-domain logit scale
    const int meta16 = J.meta16;

    float m[GM], l[GM], sws[GM], spz[GM];
    float acc[GM][T::CPL];
#pragma unroll
    for (int g = 0; g < GM; ++g) {
        m[g] = -INFINITY; l[g] = 0.f; sws[g] = 0.f; spz[g] = 0.f;
#pragma unroll
        for (int j = 0; j < T::CPL; ++j) acc[g][j] = 0.f;
    }

    for (int u = r0; t0 + u * 32 < t1; u += WPH) {
        const int ub = t0 + u * 32;
        const int tk = ub + lane;
        const bool inr = tk < t1;
        const int nt = min(32, t1 - ub);
        float s[GM];

        if (is_dense) {
            // ---------------- dense QK: lane <-> token ----------------
            if (inr) {
                const float *Kb, *Vb;
                int slot;
                dense_slot(J, tc, tk, Kb, Vb, slot);
                const float4* krow = reinterpret_cast<const float4*>(Kb + (size_t)slot * kvs + (size_t)kvh * HD);
                W.vrow[lane] = Vb + (size_t)slot * kvs + (size_t)kvh * HD;
                float a[GM];
#pragma unroll
                for (int g = 0; g < GM; ++g) a[g] = 0.f;
#pragma unroll 4
                for (int c4 = 0; c4 < HD / 4; ++c4) {
                    const float4 k = krow[c4];
#pragma unroll
                    for (int g = 0; g < GM; ++g) {
                        const float4 q = reinterpret_cast<const float4*>(qk + g * HD)[c4];
                        a[g] = fmaf(q.x, k.x, a[g]);
                        a[g] = fmaf(q.y, k.y, a[g]);
                        a[g] = fmaf(q.z, k.z, a[g]);
                        a[g] = fmaf(q.w, k.w, a[g]);
                    }
                }
#pragma unroll
                for (int g = 0; g < GM; ++g) s[g] = a[g] * sc;
            } else {
#pragma unroll
                for (int g = 0; g < GM; ++g) s[g] = -INFINITY;
            }
        } else {
            // ---------------- PBS: stage words, q*scale, bias sums ----------------
            float bs[2][GM], bz[2][GM];
#pragma unroll
            for (int hf = 0; hf < 2; ++hf) {
#pragma unroll
                for (int g = 0; g < GM; ++g) { bs[hf][g] = 0.f; bz[hf][g] = 0.f; }
                const int tb = ub + hf * 16;
                if (tb < t1) {
                    const int krow = tb >> 4, mrow = tb / J.grp;
                    const uint32_t* kp = reinterpret_cast<const uint32_t*>(J.kp) + ((size_t)krow * nkv + kvh) * HD;
                    const size_t mb = ((size_t)mrow * nkv + kvh) * HD;
#pragma unroll
                    for (int j = 0; j < T::CPL; ++j) {
                        const int c = lane * T::CPL + j;
                        if (c < HD) {
                            W.kw[hf * HD + c] = __ldg(kp + c);
                            const float sv = load_meta(J.ks, mb + c, meta16);
                            const float zv = load_meta(J.kz, mb + c, meta16);
#pragma unroll
                            for (int g = 0; g < GM; ++g) {
                                const float qv = qk[g * HD + c];
                                const float v = qv * sv;
                                W.qs[(hf * HD + c) * GM + g] = v;
                                bs[hf][g] += v;
                                bz[hf][g] = fmaf(qv, zv, bz[hf][g]);
                            }
                        }
                    }
#pragma unroll
                    for (int g = 0; g < GM; ++g) {
                        bs[hf][g] = warp_sum(bs[hf][g]);
                        bz[hf][g] = warp_sum(bz[hf][g]);
                    }
                }
            }
            __syncwarp();
            // ---------------- PBS QK: lane <-> token ----------------
            const int hf = lane >> 4;
            const int rot = (21 - 2 * (lane & 15)) & 31;
            float a[GM];
#pragma unroll
            for (int g = 0; g < GM; ++g) a[g] = 0.f;
            if (inr) {
                const uint4* kw4 = reinterpret_cast<const uint4*>(W.kw + hf * HD);
                const float* qsh = W.qs + (size_t)hf * HD * GM;
#pragma unroll 2
                for (int c4 = 0; c4 < HD / 4; ++c4) {
                    const uint4 w4 = kw4[c4];
                    const uint32_t ww[4] = {w4.x, w4.y, w4.z, w4.w};
#pragma unroll
                    for (int jj = 0; jj < 4; ++jj) {
                        const float F = unpack_4pc(ww[jj], rot);
                        const float* qc = qsh + (c4 * 4 + jj) * GM;
                        if constexpr (GM % 4 == 0) {
#pragma unroll
                            for (int g4 = 0; g4 < GM / 4; ++g4) {
                                const float4 qv = reinterpret_cast<const float4*>(qc)[g4];
                                a[g4 * 4 + 0] = fmaf(qv.x, F, a[g4 * 4 + 0]);
                                a[g4 * 4 + 1] = fmaf(qv.y, F, a[g4 * 4 + 1]);
                                a[g4 * 4 + 2] = fmaf(qv.z, F, a[g4 * 4 + 2]);
                                a[g4 * 4 + 3] = fmaf(qv.w, F, a[g4 * 4 + 3]);
                            }
                        } else {
#pragma unroll
                            for (int g = 0; g < GM; ++g) a[g] = fmaf(qc[g], F, a[g]);
                        }
                    }
                }
            }
            const bool live = inr && J.ids[tk] != -1;
#pragma unroll
            for (int g = 0; g < GM; ++g) {
                const float bsg = hf ? bs[1][g] : bs[0][g];
                const float bzg = hf ? bz[1][g] : bz[0][g];
                s[g] = live ? ((a[g] - 4.0f * bsg) + bzg) * sc : -INFINITY;
            }
        }

        // ---------------- logits to scratch (mean weights) ----------------
        if (inr) {
            const int pos = is_dense ? tk : D + tk;
#pragma unroll
            for (int g = 0; g < GM; ++g)
                if (g < G) J.scores[(size_t)(kvh * G + g) * J.score_stride + pos] = s[g];
        }

        // ---------------- online softmax ----------------
        float vsc = 0.f, vzr = 0.f;
        if (!is_dense && inr) {
            const size_t mi = (size_t)tk * nkv + kvh;
            vsc = load_meta(J.vs, mi, meta16);
            vzr = load_meta(J.vz, mi, meta16);
        }
#pragma unroll
        for (int g = 0; g < GM; ++g) {
            const float mu = warp_max(s[g]);
            const float mn = fmaxf(m[g], mu);
            float alpha = 1.f, p = 0.f;
            if (mn != -INFINITY) {
                alpha = exp2f(m[g] - mn);
                p = s[g] == -INFINITY ? 0.f : exp2f(s[g] - mn);
            }
            m[g] = mn;
            l[g] = fmaf(l[g], alpha, p);
            sws[g] *= alpha;
            spz[g] *= alpha;
#pragma unroll
            for (int j = 0; j < T::CPL; ++j) acc[g][j] *= alpha;
            if (is_dense) {
                W.ws[lane * GM + g] = p;
            } else {
                const float wsv = p * vsc;
                sws[g] += wsv;
                spz[g] = fmaf(p, vzr, spz[g]);
                W.ws[lane * GM + g] = wsv;
            }
        }

        // ---------------- PV: lane <-> channels ----------------
        if (is_dense) {
            __syncwarp();
            for (int t = 0; t < nt; ++t) {
                const float* vr = W.vrow[t] + lane * T::CPL;
                float v[T::CPL];
                if constexpr (T::CPL == 4) {
                    const float4 x = ldg_stream_f4(vr);
                    v[0] = x.x; v[1] = x.y; v[2] = x.z; v[3] = x.w;
                } else if constexpr (T::CPL == 8) {
                    const float4 x = ldg_stream_f4(vr), y = ldg_stream_f4(vr + 4);
                    v[0] = x.x; v[1] = x.y; v[2] = x.z; v[3] = x.w;
                    v[4] = y.x; v[5] = y.y; v[6] = y.z; v[7] = y.w;
                } else {
#pragma unroll
                    for (int j = 0; j < T::CPL; ++j) v[j] = (lane * T::CPL + j < HD) ? __ldg(vr + j) : 0.f;
                }
#pragma unroll
                for (int g = 0; g < GM; ++g) {
                    const float p = W.ws[t * GM + g];
#pragma unroll
                    for (int j = 0; j < T::CPL; ++j) acc[g][j] = fmaf(p, v[j], acc[g][j]);
                }
            }
        } else {
#pragma unroll
            for (int i = 0; i < T::DQ; ++i) {
                const int idx = i * 32 + lane;
                const int t = idx / T::DQ, wi = idx - (idx / T::DQ) * T::DQ;
                const int tok = ub + t;
                W.vw[t * T::DQ + wi] =
                    tok < t1 ? __ldg(reinterpret_cast<const uint32_t*>(J.vp) + ((size_t)tok * nkv + kvh) * T::DQ + wi) : 0u;
            }
            __syncwarp();
            const int wsel = min(lane * T::CPL, HD - 1) / 16;
            for (int t = 0; t < nt; ++t) {
                const uint32_t w = W.vw[t * T::DQ + wsel];
                float wg[GM];
                if constexpr (GM % 4 == 0) {
#pragma unroll
                    for (int g4 = 0; g4 < GM / 4; ++g4) {
                        const float4 x = reinterpret_cast<const float4*>(W.ws + t * GM)[g4];
                        wg[g4 * 4 + 0] = x.x; wg[g4 * 4 + 1] = x.y; wg[g4 * 4 + 2] = x.z; wg[g4 * 4 + 3] = x.w;
                    }
                } else {
#pragma unroll
                    for (int g = 0; g < GM; ++g) wg[g] = W.ws[t * GM + g];
                }
#pragma unroll
                for (int j = 0; j < T::CPL; ++j) {
                    const int bit = 2 * ((lane * T::CPL + j) & 15);
                    const float F = unpack_4pc(w, (21 - bit) & 31);
#pragma unroll
                    for (int g = 0; g < GM; ++g) acc[g][j] = fmaf(wg[g], F, acc[g][j]);
                }
            }
        }
        __syncwarp();
    }

    // ---- per-warp totals: l, and for packed V the bias terms ----
#pragma unroll
    for (int g = 0; g < GM; ++g) {
        l[g] = warp_sum(l[g]);
        if (!is_dense) {
            const float SW = warp_sum(sws[g]);
            const float SZ = warp_sum(spz[g]);
#pragma unroll
            for (int j = 0; j < T::CPL; ++j) acc[g][j] = (acc[g][j] - 4.0f * SW) + SZ;
        }
    }

    const int chunk = blockIdx.x;
    if (WPH == 1) {
#pragma unroll
        for (int g = 0; g < GM; ++g) {
            if (g >= G) break;
            const size_t qh = (size_t)kvh * G + g;
            const size_t pi = (size_t)chunk * nq + qh;
            if (lane == 0) {
                J.part_ml[pi * 2 + 0] = m[g];
                J.part_ml[pi * 2 + 1] = l[g];
            }
#pragma unroll
            for (int j = 0; j < T::CPL; ++j) {
                const int c = lane * T::CPL + j;
                if (c < HD) J.part_acc[pi * HD + c] = acc[g][j];
            }
        }
        return;
    }
    // ---- merge the WPH warps that share a kv head ----
    __syncthreads();
    float* mb = reinterpret_cast<float*>(smem + (size_t)HG * GM * HD * 4);
    float* mine = mb + (size_t)warp * GM * (HD + 2);
#pragma unroll
    for (int g = 0; g < GM; ++g) {
        if (lane == 0) {
            mine[g * (HD + 2) + 0] = m[g];
            mine[g * (HD + 2) + 1] = l[g];
        }
#pragma unroll
        for (int j = 0; j < T::CPL; ++j) {
            const int c = lane * T::CPL + j;
            if (c < HD) mine[g * (HD + 2) + 2 + c] = acc[g][j];
        }
    }
    __syncthreads();
    if (r0 != 0) return;
    for (int g = 0; g < G && g < GM; ++g) {
        float M = -INFINITY;
        for (int r = 0; r < WPH; ++r) M = fmaxf(M, mb[(size_t)(r * HG + kvl) * GM * (HD + 2) + g * (HD + 2)]);
        float Ls = 0.f;
        float o[T::CPL];
#pragma unroll
        for (int j = 0; j < T::CPL; ++j) o[j] = 0.f;
        for (int r = 0; r < WPH; ++r) {
            const float* src = mb + (size_t)(r * HG + kvl) * GM * (HD + 2) + g * (HD + 2);
            const float mr = src[0];
            if (mr == -INFINITY) continue;
            const float f = exp2f(mr - M);
            Ls = fmaf(src[1], f, Ls);
#pragma unroll
            for (int j = 0; j < T::CPL; ++j) {
                const int c = lane * T::CPL + j;
                if (c < HD) o[j] = fmaf(src[2 + c], f, o[j]);
            }
        }
        const size_t pi = (size_t)chunk * nq + (size_t)kvh * G + g;
        if (lane == 0) {
            J.part_ml[pi * 2 + 0] = M;
            J.part_ml[pi * 2 + 1] = Ls;
        }
#pragma unroll
        for (int j = 0; j < T::CPL; ++j) {
            const int c = lane * T::CPL + j;
            if (c < HD) J.part_acc[pi * HD + c] = o[j];
        }
    }
}

// ---------------------------------------------------------------------------
// merge + mean weights + score feedback
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(NT) k_attn_finalize(const __grid_constant__ AttnLaunch L) {
    extern __shared__ __align__(16) unsigned char smem[];
    __shared__ JobDesc Js;
    __shared__ TierCounts Ts;
    const int job = blockIdx.y;
    if (threadIdx.x == 0) {
        Js = L.jobs[job] ? *L.jobs[job] : L.inline_job;
        Ts = resolve_counts(Js);
    }
    __syncthreads();
    const JobDesc& J = Js;
    const TierCounts tc = Ts;
    const int nq = J.nq, HD = J.hd;
    const int D = tc.n0 + tc.n1 + tc.n2;
    const int ntok = tc.nblk * J.grp;
    const int T = D + ntok;
    const int nd_act = ceil_div(D, L.DC), np_act = ceil_div(ntok, L.PC);
    const int nch = nd_act + np_act;
    float* Ms = reinterpret_cast<float*>(smem);
    float* Ls = Ms + nq;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    for (int h = warp; h < nq; h += NW) {
        float M = -INFINITY;
        for (int i = lane; i < nch; i += 32) {
            const int ci = i < nd_act ? i : L.nd + (i - nd_act);
            M = fmaxf(M, J.part_ml[((size_t)ci * nq + h) * 2]);
        }
        M = warp_max(M);
        float S = 0.f;
        if (M != -INFINITY) {
            for (int i = lane; i < nch; i += 32) {
                const int ci = i < nd_act ? i : L.nd + (i - nd_act);
                const float mi = J.part_ml[((size_t)ci * nq + h) * 2];
                if (mi != -INFINITY) S = fmaf(J.part_ml[((size_t)ci * nq + h) * 2 + 1], exp2f(mi - M), S);
            }
        }
        S = warp_sum(S);
        if (lane == 0) {
            Ms[h] = M;
            Ls[h] = S > 0.f ? S : 1.0f;  // row_sum_exp fallback (fused_attn_avx2.cpp:261)
        }
    }
    __syncthreads();

    // ---- attention output: heads blockIdx.x, blockIdx.x + nfin, ... ----
    float* out = L.out[job];
    for (int h = blockIdx.x; h < nq; h += L.nfin) {
        const float M = Ms[h], inv = 1.0f / Ls[h];
        for (int c = threadIdx.x; c < HD; c += NT) {
            float o = 0.f;
            if (M != -INFINITY) {
                for (int i = 0; i < nch; ++i) {
                    const int ci = i < nd_act ? i : L.nd + (i - nd_act);
                    const float mi = J.part_ml[((size_t)ci * nq + h) * 2];
                    if (mi == -INFINITY) continue;
                    o = fmaf(J.part_acc[((size_t)ci * nq + h) * HD + c], exp2f(mi - M), o);
                }
            }
            out[(size_t)h * HD + c] = o * inv;
        }
    }

    // ---- mean attention weights over heads, score feedback ----
    float* mw = L.mw[job];
    const int p0 = blockIdx.x * L.FT, p1 = min(T, p0 + L.FT);
    for (int pos = p0 + threadIdx.x; pos < p1; pos += NT) {
        float sw = 0.f;
        for (int h = 0; h < nq; ++h) {
            const float s = J.scores[(size_t)h * J.score_stride + pos];
            if (s != -INFINITY) sw += exp2f(s - Ms[h]) / Ls[h];
        }
        const float w = sw / (float)nq;
        if (mw) mw[pos] = w;
        if (J.g) {
            long long id;
            if (pos < tc.n0) {
                id = pos;
            } else if (pos < tc.n0 + tc.n1) {
                const int i = pos - tc.n0;
                id = J.hh_ids[i];
                if (id >= 0 && id < J.msl) {
                    const float nv = fmaf(J.decay, J.g[id], w);
                    J.g[id] = nv;
                    J.hh_scores[i] = nv;
                }
                continue;
            } else if (pos < D) {
                id = (long long)tc.total - tc.n2 + (pos - tc.n0 - tc.n1);
            } else {
                id = J.ids[pos - D];
            }
            if (id >= 0 && id < J.msl) J.g[id] = fmaf(J.decay, J.g[id], w);
        }
    }
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
int attn_max_chunks(int dense_cap, int pbs_tok_cap) { return ceil_div(dense_cap, 64) + ceil_div(pbs_tok_cap, 64) + 2; }

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
    L.HG = (nkv % 8 == 0) ? 8 : (nkv % 4 == 0) ? 4 : (nkv % 2 == 0) ? 2 : 1;
    L.nhg = nkv / L.HG;
    // Aim for about four resident CTAs' worth of work per SM across the launch.
    const long long work = (long long)L.njobs * L.nhg * ((long long)dense_cap + pbs_tok_cap);
    long long cs = work / (4LL * 148);
    cs = (cs + 31) / 32 * 32;
    cs = std::max(64LL, std::min(2048LL, cs));
    L.DC = (int)cs;
    L.PC = (int)cs;
    L.nd = ceil_div(dense_cap, L.DC);
    L.np = ceil_div(pbs_tok_cap, L.PC);
    L.FT = 1024;
    L.nfin = std::max(1, ceil_div(dense_cap + pbs_tok_cap, L.FT));
    return TT_OK;
}

template <int HD, int GM>
static tt_status launch_partial_t(const AttnLaunch& L, cudaStream_t st) {
    const size_t sm = SmemPlan<HD, GM>::bytes(L.HG);
    static bool configured[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (!configured[dev & 63]) {
        cudaError_t e = cudaFuncSetAttribute(k_attn_partial<HD, GM>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (int)SmemPlan<HD, GM>::bytes(8));
        if (e != cudaSuccess) return check_cuda(e, "cudaFuncSetAttribute(k_attn_partial)");
        configured[dev & 63] = true;
    }
    dim3 grid(L.nd + L.np, L.njobs * L.nhg);
    const int ps = prof_begin(1, st);
    k_attn_partial<HD, GM><<<grid, NT, sm, st>>>(L);
    prof_end(ps, st);
    return check_launch("k_attn_partial");
}

template <int HD>
static tt_status launch_partial_hd(const AttnLaunch& L, cudaStream_t st) {
    switch (pick_gm(L.G)) {
        case 1: return launch_partial_t<HD, 1>(L, st);
        case 2: return launch_partial_t<HD, 2>(L, st);
        case 4: return launch_partial_t<HD, 4>(L, st);
        case 8:
            if constexpr (HD <= 128) return launch_partial_t<HD, 8>(L, st);
            return set_error(TT_ERR_UNSUPPORTED, "head_dim 256 supports at most 4 query heads per kv head");
    }
    return set_error(TT_ERR_UNSUPPORTED, "unsupported GQA ratio");
}

// L.inline_job.hd / .nq must be set for engine batches too (they select the
// kernel instantiation and the finalize shared memory).
tt_status launch_attention(const AttnLaunch& L, cudaStream_t st) {
    if (L.nd + L.np > 0) {
        tt_status s;
        switch (L.inline_job.hd) {  // callers always fill inline_job.hd/nq (also for engine batches)
            case 16: s = launch_partial_hd<16>(L, st); break;
            case 32: s = launch_partial_hd<32>(L, st); break;
            case 64: s = launch_partial_hd<64>(L, st); break;
            case 128: s = launch_partial_hd<128>(L, st); break;
            case 256: s = launch_partial_hd<256>(L, st); break;
            default: return set_error(TT_ERR_UNSUPPORTED, "unsupported head_dim");
        }
        if (s != TT_OK) return s;
    }
    dim3 grid(L.nfin, L.njobs);
    const int ps = prof_begin(2, st);
    k_attn_finalize<<<grid, NT, (size_t)2 * L.inline_job.nq * sizeof(float), st>>>(L);
    prof_end(ps, st);
    return check_launch("k_attn_finalize");
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
        (num_blocks > 0 && (!aligned16(PBS_K_Packed) || !aligned16(PBS_V_Packed))))
        return set_error(TT_ERR_INVALID_ARGUMENT, "Q, dense_K, dense_V and packed PBS buffers must be 16-byte aligned.");

    AttnLaunch L;
    memset(&L, 0, sizeof(L));
    L.njobs = 1;
    const int ntok = num_blocks * k_group_size;
    tt_status s = plan_attention(L, num_q_heads, num_kv_heads, head_dim, dense_count, ntok);
    if (s != TT_OK) return s;
    int dev = 0;
    s = check_cuda(cudaGetDevice(&dev), "cudaGetDevice");
    if (s != TT_OK) return s;
    const int T = dense_count + ntok;
    const int maxch = L.nd + L.np;
    const size_t stride = (size_t)std::max(T, 1);
    const size_t need = (size_t)maxch * num_q_heads * (head_dim + 2) + (size_t)num_q_heads * stride + 64;
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
    J.part_acc = ws + (size_t)maxch * num_q_heads * 2;
    J.scores = J.part_acc + (size_t)maxch * num_q_heads * head_dim;
    J.score_stride = (int)stride;
    J.max_chunks = maxch;
    J.g = nullptr; J.hh_scores = nullptr; J.hh_ids = nullptr; J.decay = 0.f; J.msl = 0;
    L.jobs[0] = nullptr;
    L.Q[0] = Q;
    L.out[0] = attn_output;
    L.mw[0] = mean_attn_weights;
    return launch_attention(L, (cudaStream_t)stream);
}
