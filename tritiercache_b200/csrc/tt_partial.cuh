// tt_partial.cuh -- k_attn_packed: split-KV decode attention over one chunk
// of packed (2-bit) tokens for one kv-head group, plus what it shares with the
// dense kernel (tt_dense.cuh): small PTX helpers, the per-job chunk merge in
// the last CTA.  Included by tt_attn.cu only.
//
// Head dims 64 / 128 with fp16 metadata run the tensor-core unit
// (tt_pbs_mma.cuh: mma.sync f16, per-warp cp.async pipelines); the rest run
// the SIMT unit described here.  Its chunks stream through shared memory in
// stages of 256 (token, kv-head) pairs with 1-D TMA bulk copies
// (cp.async.bulk ... mbarrier::complete_tx), two stages in flight.  Every mbarrier wait is bounded: on expiry the CTA
// records TT_ERR_TIMEOUT in the device error word, drains its own copies
// (again bounded) and returns.  Every copy lands in the issuing CTA's own
// shared memory; no cluster launch.
//
// Per 32-token unit and kv head (one warp):
//   QK lane <-> token:  score = sum_c qs_c*(4+code) - 4*sum qs + sum q*zero,
//       qs = q*scale per block and channel (tabled in shared memory), the
//       2-bit code rotated into a float's mantissa (unpack_4pc), two query
//       heads per packed f32x2 FMA.
//   PV lane <-> channels: acc += (p*vscale) * (4+code), two channels per
//       f32x2 FMA; the running sums of p*vscale and p*vzero fold the
//       zero/offset back in at the end.
#pragma once
#include "tt_attn.cuh"
#include "tt_weights.cuh"

namespace tt {

constexpr int NT = 256;
constexpr int NW = NT / TT_WARP;
constexpr int NSTAGE = 2;    // stages in flight, SIMT packed unit
constexpr float kLog2e = 1.4426950408889634f;

__device__ int g_device_error = 0;  // first device-side error code (tt_status), cleared by the host

template <int HD>
struct HDT {
    static constexpr int CPL = HD >= 32 ? HD / 32 : 1;  // channels per lane in PV
    static constexpr int DQ = HD / 16;                  // packed V words per (token, head)
};

// ---------------------------------------------------------------------------
// small PTX helpers
// ---------------------------------------------------------------------------
typedef unsigned long long u64;

__device__ __forceinline__ u64 f2pack(float lo, float hi) {
    u64 r;
    asm("mov.b64 %0, {%1,%2};" : "=l"(r) : "f"(lo), "f"(hi));
    return r;
}
__device__ __forceinline__ float2 f2unpack(u64 r) {
    float2 v;
    asm("mov.b64 {%0,%1}, %2;" : "=f"(v.x), "=f"(v.y) : "l"(r));
    return v;
}
__device__ __forceinline__ u64 ffma2(u64 a, u64 b, u64 c) {
    u64 d;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
    return d;
}
__device__ __forceinline__ u64 fmul2(u64 a, u64 b) {
    u64 d;
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}
__device__ __forceinline__ float warp_max_redux(float v) {
    float m;
    asm volatile("redux.sync.max.f32 %0, %1, 0xffffffff;" : "=f"(m) : "f"(v));
    return m;
}

// 4 + code as a float, code = the 2-bit field of `w` at bit `bit` (rot = (21 - bit) & 31):
// rotate the field to mantissa bits 21-22 and set the exponent of [4, 8).
__device__ __forceinline__ float unpack_4pc(uint32_t w, int rot) {
    return __uint_as_float((__funnelshift_l(w, w, rot) & 0x00600000u) | 0x40800000u);
}

__device__ __forceinline__ uint32_t smem_addr(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_fence_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t phase) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}"
        : "=r"(ok)
        : "r"(smem_addr(bar)), "r"(phase)
        : "memory");
    return ok != 0;
}
// Bounded wait: about 2^20 polls (each try_wait may itself suspend briefly).
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t phase) {
    for (int i = 0; i < (1 << 20); ++i)
        if (mbar_try_wait(bar, phase)) return true;
    return false;
}
// L2 policies: the tiers stream through once (evict first), the logits the
// attention writes are read again by the weights pass (evict last, so that
// as many of them as fit stay in L2).
__device__ __forceinline__ uint64_t l2_evict_first() {
    uint64_t p;
    asm("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
    return p;
}
__device__ __forceinline__ uint64_t l2_evict_last() {
    uint64_t p;
    asm("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
    return p;
}
// A logit store (kept in L2 for the weights pass).
__device__ __forceinline__ void st_logit(float* p, float v) {
    asm volatile("st.global.L2::cache_hint.f32 [%0], %1, %2;" ::"l"(p), "f"(v), "l"(l2_evict_last()) : "memory");
}
// 16-byte asynchronous copy global -> shared (L2 only; cp.async groups).  No
// eviction hint: a policy register per copy costs the tensor-core unit spills.
__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_addr(dst)), "l"(src) : "memory");
}
// 1-D bulk copy global -> this CTA's shared memory, completion counted on `bar` (streaming).
__device__ __forceinline__ void tma_load_1d(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::
            "r"(smem_addr(dst)),
        "l"(src), "r"(bytes), "r"(smem_addr(bar)), "l"(l2_evict_first())
        : "memory");
}

// ---------------------------------------------------------------------------
// shared-memory plan
// ---------------------------------------------------------------------------
__host__ __device__ __forceinline__ int align_up(int x, int a) { return (x + a - 1) / a * a; }

// One stage holds ST = 32 * (NW / HG) tokens of the HG heads of a group
// (at most 256 (token, kv head) pairs).
__host__ __device__ __forceinline__ int stage_tokens(int HG) { return 32 * (NW / HG); }

struct StageLayout {
    int kw, ks, kz, vw, vs, vz, ids, bytes;
};
__host__ __device__ __forceinline__ StageLayout stage_layout(int HD, int mb, int HG = 8) {
    StageLayout s;
    int o = 0;
    s.kw = o; o += 16 * HD * 4;              // [ST/16 rows][HG][HD] words   (rows*HG = 16)
    s.ks = o; o += align_up(16 * HD * mb, 16);  // [blocks][HG][HD]        (blocks*HG <= 16)
    s.kz = o; o += align_up(16 * HD * mb, 16);
    s.vw = o;                                // [ST][HG][DQ] (+ pad per token)
    o += 256 * (HD / 16) * 4;
    s.vs = o; o += align_up(256 * mb, 16);   // [ST][HG]
    s.vz = o; o += align_up(256 * mb, 16);
    s.ids = o; o += 256 * 8;                 // [ST] (ST <= 256)
    s.bytes = align_up(o, 128);
    return s;
}

// Per-warp shared memory of the SIMT packed unit.
template <int HD, int GM>
struct WarpArea {
    static constexpr int qs = 2 * HD * GM * 4;  // q*scale table [half][HD][GM]
    static constexpr int ws = 32 * GM * 8;      // [token][GM] (w, w) pairs
    static constexpr int bias = 2 * 2 * GM * 4; // [half][sum qs | sum q*z][GM]
    static constexpr int bytes = qs + ws + bias;
};

template <int HD, int GM>
__host__ __device__ __forceinline__ size_t partial_smem_bytes(int HG, int mb) {
    const size_t q = (size_t)align_up(HG * GM * HD * 4, 128);
    const size_t body = (size_t)NSTAGE * stage_layout(HD, mb, HG).bytes + (size_t)NW * WarpArea<HD, GM>::bytes;
    const size_t merge = (size_t)NW * GM * (HD + 2) * 4;
    return q + (body > merge ? body : merge);
}

// K/V tier rows and slot of local dense position i (tt_attn.cuh numbering).
__device__ __forceinline__ void dense_slot(const JobDesc& J, const TierCounts& tc, int i, int r, int w, const float*& Kb,
                                           const float*& Vb, int& slot) {
    const int tier = dense_local_slot(tc, i, r, w, slot);
    Kb = tier == 0 ? J.K0 : tier == 1 ? J.K1 : J.K2;
    Vb = tier == 0 ? J.V0 : tier == 1 ? J.V1 : J.V2;
}

// Per-warp online-softmax state.  acc holds channel pairs (lane owns CPL channels).
template <int HD, int GM>
struct WarpState {
    static constexpr int CPL = HDT<HD>::CPL;
    static constexpr int NP = CPL >= 2 ? CPL / 2 : 1;
    float m[GM], l[GM], sws[GM], spz[GM];
    u64 acc2[GM][NP];   // CPL >= 2
    float acc1[GM];     // CPL == 1
    __device__ __forceinline__ void init() {
#pragma unroll
        for (int g = 0; g < GM; ++g) {
            m[g] = -INFINITY; l[g] = 0.f; sws[g] = 0.f; spz[g] = 0.f; acc1[g] = 0.f;
#pragma unroll
            for (int p = 0; p < NP; ++p) acc2[g][p] = 0ull;
        }
    }
};

// online softmax update for one 32-token unit; returns p[g] for this lane's token
template <int HD, int GM>
__device__ __forceinline__ void softmax_update(WarpState<HD, GM>& S, const float (&s)[GM], float (&p)[GM]) {
#pragma unroll
    for (int g = 0; g < GM; ++g) {
        const float mu = warp_max_redux(s[g]);
        const float mn = fmaxf(S.m[g], mu);
        float alpha = 1.f, pv = 0.f;
        if (mn != -INFINITY) {
            alpha = exp2f(S.m[g] - mn);
            pv = s[g] == -INFINITY ? 0.f : exp2f(s[g] - mn);
        }
        S.m[g] = mn;
        S.l[g] = fmaf(S.l[g], alpha, pv);
        S.sws[g] *= alpha;
        S.spz[g] *= alpha;
        if constexpr (WarpState<HD, GM>::CPL >= 2) {
            const u64 a2 = f2pack(alpha, alpha);
#pragma unroll
            for (int q = 0; q < WarpState<HD, GM>::NP; ++q) S.acc2[g][q] = fmul2(S.acc2[g][q], a2);
        } else {
            S.acc1[g] *= alpha;
        }
        p[g] = pv;
    }
}

// Sum of v[0..N) over the warp, scattered: lane l ends with the total of value
// (l >> (5 - log2 N)) ... returned through `out` written to shared memory.
template <int N>
__device__ __forceinline__ void warp_reduce_scatter_to_smem(float (&v)[N], float* out, int lane) {
    static_assert((N & (N - 1)) == 0 && N <= 32, "power of two");
    int cnt = N;
    int idx = 0;
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
            if (up) idx += half;
            cnt = half;
        } else {
            v[0] += __shfl_xor_sync(0xffffffffu, v[0], o);
        }
    }
    // every lane holds the full total of value idx; the lowest such lane stores it
    const int lanes_per_value = 32 / N;
    if ((lane & (lanes_per_value - 1)) == 0) out[idx] = v[0];
}

// the GM (w, w) pairs of one token from the ws table, 16 bytes per load
template <int GM>
__device__ __forceinline__ void load_wrow(const u64* wt, u64 (&w)[GM]) {
    if constexpr (GM % 2 == 0) {
#pragma unroll
        for (int g2 = 0; g2 < GM / 2; ++g2) {
            const ulonglong2 x = reinterpret_cast<const ulonglong2*>(wt)[g2];
            w[2 * g2] = x.x;
            w[2 * g2 + 1] = x.y;
        }
    } else {
        w[0] = wt[0];
    }
}

// ---------------------------------------------------------------------------
// packed chunk
// ---------------------------------------------------------------------------
template <int HD, int GM>
__device__ __forceinline__ void pbs_issue_stage(const JobDesc& J, int HG, int hg, int t0, int t1, int s,
                                                unsigned char* stages, const StageLayout& SL, uint64_t* bars,
                                                int lane, int rank, int world) {
    constexpr int DQ = HDT<HD>::DQ;
    const int ST = stage_tokens(HG);
    const int nt = min(ST, t1 - (t0 + s * ST));
    const int s0 = packed_global(t0 + s * ST, rank, world);  // a stage lies inside one ownership granule
    const int grp = J.grp, nkv = J.nkv, h0 = hg * HG;
    // Every copy below starts 16-byte aligned and moves a multiple of 16 bytes:
    // HG == nkv gives one contiguous run per region; otherwise HG == 8 and the
    // per-row / per-block / per-token slices are HG*HD*4, HG*HD*mb, HG*HD/4 and
    // HG*mb >= 16 bytes (plan_attention guarantees one of the two).
    const int mb = J.meta16 ? 2 : 4;
    const int rows = nt / 16, blks = nt / grp;
    unsigned char* buf = stages + (size_t)(s % NSTAGE) * SL.bytes;
    uint64_t* bar = &bars[s % NSTAGE];
    const uint32_t bytes = (uint32_t)rows * HG * HD * 4 + 2u * blks * HG * HD * mb + (uint32_t)nt * HG * DQ * 4 +
                           2u * nt * HG * mb + (uint32_t)nt * 8;
    if (lane == 0) mbar_expect_tx(bar, bytes);
    __syncwarp();
    const char* kp = reinterpret_cast<const char*>(J.kp);
    const char* ks = reinterpret_cast<const char*>(J.ks);
    const char* kz = reinterpret_cast<const char*>(J.kz);
    const char* vp = reinterpret_cast<const char*>(J.vp);
    const char* vs = reinterpret_cast<const char*>(J.vs);
    const char* vz = reinterpret_cast<const char*>(J.vz);
    const char* ids = reinterpret_cast<const char*>(J.ids);
    if (HG == nkv) {
        if (lane == 0) tma_load_1d(buf + SL.kw, kp + (size_t)(s0 / 16) * nkv * HD * 4, rows * HG * HD * 4, bar);
        if (lane == 1) tma_load_1d(buf + SL.ks, ks + (size_t)(s0 / grp) * nkv * HD * mb, blks * HG * HD * mb, bar);
        if (lane == 2) tma_load_1d(buf + SL.kz, kz + (size_t)(s0 / grp) * nkv * HD * mb, blks * HG * HD * mb, bar);
        if (lane == 3) tma_load_1d(buf + SL.vw, vp + (size_t)s0 * nkv * DQ * 4, nt * HG * DQ * 4, bar);
        if (lane == 4) tma_load_1d(buf + SL.vs, vs + (size_t)s0 * nkv * mb, nt * HG * mb, bar);
        if (lane == 5) tma_load_1d(buf + SL.vz, vz + (size_t)s0 * nkv * mb, nt * HG * mb, bar);
        if (lane == 6) tma_load_1d(buf + SL.ids, ids + (size_t)s0 * 8, nt * 8, bar);
    } else {
        for (int i = lane; i < rows; i += 32)
            tma_load_1d(buf + SL.kw + (size_t)i * HG * HD * 4, kp + ((size_t)(s0 / 16 + i) * nkv + h0) * HD * 4,
                        HG * HD * 4, bar);
        for (int i = lane; i < blks; i += 32) {
            const size_t off = ((size_t)(s0 / grp + i) * nkv + h0) * HD * mb;
            tma_load_1d(buf + SL.ks + (size_t)i * HG * HD * mb, ks + off, HG * HD * mb, bar);
            tma_load_1d(buf + SL.kz + (size_t)i * HG * HD * mb, kz + off, HG * HD * mb, bar);
        }
        for (int i = lane; i < nt; i += 32) {
            tma_load_1d(buf + SL.vw + (size_t)i * HG * DQ * 4, vp + ((size_t)(s0 + i) * nkv + h0) * DQ * 4,
                        HG * DQ * 4, bar);
            const size_t mo = ((size_t)(s0 + i) * nkv + h0) * mb;
            tma_load_1d(buf + SL.vs + (size_t)i * HG * mb, vs + mo, HG * mb, bar);
            tma_load_1d(buf + SL.vz + (size_t)i * HG * mb, vz + mo, HG * mb, bar);
        }
        if (lane == 0) tma_load_1d(buf + SL.ids, ids + (size_t)s0 * 8, nt * 8, bar);
    }
}

template <int HD, int GM>
__device__ __forceinline__ void pbs_unit(const JobDesc& J, int HG, int G, int kvl, int kvh, int lane, int D,
                                         const unsigned char* buf, const StageLayout& SL, int s0, int nt, int r,
                                         const float* qk, unsigned char* wa, float sc, WarpState<HD, GM>& S) {
    constexpr int CPL = HDT<HD>::CPL, DQ = HDT<HD>::DQ;
    using WA = WarpArea<HD, GM>;
    float* qs_tab = reinterpret_cast<float*>(wa);
    u64* ws_tab = reinterpret_cast<u64*>(wa + WA::qs);
    float* bias = reinterpret_cast<float*>(wa + WA::qs + WA::ws);
    const int grp = J.grp;
    const int mb = J.meta16 ? 2 : 4;
    const int ub = r * 32;  // unit start within the stage
    const uint32_t* kw_s = reinterpret_cast<const uint32_t*>(buf + SL.kw);
    const unsigned char* ks_s = buf + SL.ks;
    const unsigned char* kz_s = buf + SL.kz;
    const uint32_t* vw_s = reinterpret_cast<const uint32_t*>(buf + SL.vw);
    const unsigned char* vs_s = buf + SL.vs;
    const unsigned char* vz_s = buf + SL.vz;
    const int64_t* ids_s = reinterpret_cast<const int64_t*>(buf + SL.ids);

    // ---- qs = q*scale tables and per-block bias sums ----
    // lane <-> channels lane, lane+32, ...: consecutive lanes touch consecutive
    // shared-memory words (metadata, q) and write whole GM-wide table rows.
    float part[4 * GM];  // [half][qs-sum | qz-sum][g]
#pragma unroll
    for (int i = 0; i < 4 * GM; ++i) part[i] = 0.f;
#pragma unroll
    for (int hf = 0; hf < 2; ++hf) {
        const int tb = ub + hf * 16;
        if (tb < nt) {
            const int mblk = tb / grp;
            const size_t mo = ((size_t)mblk * HG + kvl) * HD;
#pragma unroll
            for (int j = 0; j < CPL; ++j) {
                const int c = lane + 32 * j;
                if (c < HD) {
                    const float sv = load_meta(ks_s, mo + c, mb == 2);
                    const float zv = load_meta(kz_s, mo + c, mb == 2);
                    float v[GM];
#pragma unroll
                    for (int g = 0; g < GM; ++g) {
                        const float qv = qk[g * HD + c];
                        v[g] = qv * sv;
                        part[(hf * 2 + 0) * GM + g] += v[g];
                        part[(hf * 2 + 1) * GM + g] = fmaf(qv, zv, part[(hf * 2 + 1) * GM + g]);
                    }
                    float* dst = qs_tab + (size_t)(hf * HD + c) * GM;
                    if constexpr (GM % 4 == 0) {
#pragma unroll
                        for (int g4 = 0; g4 < GM / 4; ++g4)
                            reinterpret_cast<float4*>(dst)[g4] =
                                make_float4(v[4 * g4], v[4 * g4 + 1], v[4 * g4 + 2], v[4 * g4 + 3]);
                    } else if constexpr (GM == 2) {
                        *reinterpret_cast<float2*>(dst) = make_float2(v[0], v[1]);
                    } else {
                        dst[0] = v[0];
                    }
                }
            }
        }
    }
    warp_reduce_scatter_to_smem<4 * GM>(part, bias, lane);
    __syncwarp();

    // ---- QK: lane <-> token ----
    const int tl = ub + lane;  // token within the stage
    const bool inr = tl < nt;
    const int hf = lane >> 4;
    const int rot = (21 - 2 * (lane & 15)) & 31;
    float s[GM];
    {
        const int row = inr ? (tl >> 4) : (ub >> 4);
        const uint4* kw4 = reinterpret_cast<const uint4*>(kw_s + ((size_t)row * HG + kvl) * HD);
        const float* qsh = qs_tab + (size_t)hf * HD * GM;
        // two accumulator sets (even / odd channel quads) for independent FMA chains
        constexpr int NG2 = GM >= 2 ? GM / 2 : 1;
        u64 a2[2][NG2];
        float a1[2] = {0.f, 0.f};
#pragma unroll
        for (int e = 0; e < 2; ++e)
#pragma unroll
            for (int g2 = 0; g2 < NG2; ++g2) a2[e][g2] = 0ull;
#pragma unroll 2
        for (int c4 = 0; c4 < HD / 4; ++c4) {
            const uint4 w4 = kw4[c4];
            const uint32_t ww[4] = {w4.x, w4.y, w4.z, w4.w};
            const int e = c4 & 1;
#pragma unroll
            for (int jj = 0; jj < 4; ++jj) {
                const float F = unpack_4pc(ww[jj], rot);
                const float* qc = qsh + (c4 * 4 + jj) * GM;
                if constexpr (GM == 1) {
                    a1[e] = fmaf(qc[0], F, a1[e]);
                } else {
                    const u64 FF = f2pack(F, F);
                    if constexpr (GM % 4 == 0) {
#pragma unroll
                        for (int g4 = 0; g4 < GM / 4; ++g4) {
                            const ulonglong2 q4 = reinterpret_cast<const ulonglong2*>(qc)[g4];
                            a2[e][2 * g4] = ffma2(q4.x, FF, a2[e][2 * g4]);
                            a2[e][2 * g4 + 1] = ffma2(q4.y, FF, a2[e][2 * g4 + 1]);
                        }
                    } else {
#pragma unroll
                        for (int g2 = 0; g2 < NG2; ++g2)
                            a2[e][g2] = ffma2(*reinterpret_cast<const u64*>(qc + 2 * g2), FF, a2[e][g2]);
                    }
                }
            }
        }
        const bool live = inr && ids_s[tl] != -1;
        const float* bsh = bias + hf * 2 * GM;
#pragma unroll
        for (int g = 0; g < GM; ++g) {
            float a;
            if constexpr (GM == 1) {
                a = a1[0] + a1[1];
            } else {
                const float2 v0 = f2unpack(a2[0][g / 2]), v1 = f2unpack(a2[1][g / 2]);
                a = (g & 1) ? (v0.y + v1.y) : (v0.x + v1.x);
            }
            s[g] = live ? ((a - 4.0f * bsh[g]) + bsh[GM + g]) * sc : -INFINITY;
        }
    }
    // ---- logits to scratch ----
    if (inr) {
        const int pos = D + s0 + tl;
#pragma unroll
        for (int g = 0; g < GM; ++g)
            if (g < G) st_logit(J.scores + (size_t)(kvh * G + g) * J.score_stride + pos, s[g]);
    }
    // ---- softmax, V weights ----
    float p[GM];
    softmax_update<HD, GM>(S, s, p);
    float vsc = 0.f, vzr = 0.f;
    if (inr) {
        vsc = load_meta(vs_s, (size_t)tl * HG + kvl, mb == 2);
        vzr = load_meta(vz_s, (size_t)tl * HG + kvl, mb == 2);
    }
    {
        u64 wrow[GM];
#pragma unroll
        for (int g = 0; g < GM; ++g) {
            const float w = p[g] * vsc;
            S.sws[g] += w;
            S.spz[g] = fmaf(p[g], vzr, S.spz[g]);
            wrow[g] = f2pack(w, w);
        }
        u64* dst = ws_tab + lane * GM;
        if constexpr (GM % 2 == 0) {
#pragma unroll
            for (int g2 = 0; g2 < GM / 2; ++g2) reinterpret_cast<ulonglong2*>(dst)[g2] = make_ulonglong2(wrow[2 * g2], wrow[2 * g2 + 1]);
        } else {
            dst[0] = wrow[0];
        }
    }
    __syncwarp();
    // ---- PV: lane <-> channels ----
    const int ntu = min(32, nt - ub);
    const int c0 = min(lane * CPL, HD - 1);
    const int wi = c0 / 16;
    int rotc[CPL];
#pragma unroll
    for (int j = 0; j < CPL; ++j) rotc[j] = (21 - 2 * ((c0 + j) & 15)) & 31;
#pragma unroll 2
    for (int t = 0; t < ntu; ++t) {
        const uint32_t w = vw_s[((size_t)(ub + t) * HG + kvl) * DQ + wi];
        const u64* wt = ws_tab + t * GM;
        u64 wrow[GM];
        load_wrow<GM>(wt, wrow);
        if constexpr (CPL >= 2) {
            u64 F2[CPL / 2];
#pragma unroll
            for (int q = 0; q < CPL / 2; ++q) F2[q] = f2pack(unpack_4pc(w, rotc[2 * q]), unpack_4pc(w, rotc[2 * q + 1]));
#pragma unroll
            for (int g = 0; g < GM; ++g) {
                const u64 wg = wrow[g];
#pragma unroll
                for (int q = 0; q < CPL / 2; ++q) S.acc2[g][q] = ffma2(wg, F2[q], S.acc2[g][q]);
            }
        } else {
            const float F = unpack_4pc(w, rotc[0]);
#pragma unroll
            for (int g = 0; g < GM; ++g) S.acc1[g] = fmaf(f2unpack(wt[g]).x, F, S.acc1[g]);
        }
    }
    __syncwarp();
}

}  // namespace tt

#include "tt_pbs_mma.cuh"

namespace tt {

// ---------------------------------------------------------------------------
// the kernel
// ---------------------------------------------------------------------------
// Writes one warp's (m, l, output row) for query head g of its kv head: to the
// chunk's partials directly (one warp per kv head) or to the merge buffer.
__device__ __forceinline__ size_t part_index(const JobDesc& J, int chunk, int kvh, int G, int g) {
    return (size_t)chunk * J.nq + (size_t)kvh * G + g;
}

// Merges the WPH warps that share a kv head (their rows are in mbuf,
// [warp][GM][m, l, HD]) and writes the chunk's partials; run by warps r0 == 0.
template <int HD, int GM>
__device__ __forceinline__ void merge_warps(const JobDesc& J, const float* mbuf, int chunk, int kvh, int kvl, int HG,
                                            int WPH, int G, int lane) {
    constexpr int CPL = HDT<HD>::CPL;
    for (int g = 0; g < G && g < GM; ++g) {
        float M = -INFINITY;
        for (int r = 0; r < WPH; ++r) M = fmaxf(M, mbuf[(size_t)(r * HG + kvl) * GM * (HD + 2) + g * (HD + 2)]);
        float Ls = 0.f;
        float o[CPL];
#pragma unroll
        for (int j = 0; j < CPL; ++j) o[j] = 0.f;
        for (int r = 0; r < WPH; ++r) {
            const float* src = mbuf + (size_t)(r * HG + kvl) * GM * (HD + 2) + g * (HD + 2);
            const float mr = src[0];
            if (mr == -INFINITY) continue;
            const float f = exp2f(mr - M);
            Ls = fmaf(src[1], f, Ls);
#pragma unroll
            for (int j = 0; j < CPL; ++j) {
                const int c = lane * CPL + j;
                if (c < HD) o[j] = fmaf(src[2 + c], f, o[j]);
            }
        }
        const size_t pi = part_index(J, chunk, kvh, G, g);
        if (lane == 0) {
            J.part_ml[pi * 2 + 0] = M;
            J.part_ml[pi * 2 + 1] = Ls;
        }
#pragma unroll
        for (int j = 0; j < CPL; ++j) {
            const int c = lane * CPL + j;
            if (c < HD) J.part_acc[pi * HD + c] = o[j];
        }
    }
}

// Shared memory of k_attn_packed<HD, GM, MMA>: the SIMT kernel's plan
// (partial_smem_bytes), or for the tensor-core kernel the query rows followed
// by one MmaWarpArea per warp.
template <int HD, int GM, bool MMA>
__host__ __device__ __forceinline__ size_t kernel_smem_bytes(int HG, int mb) {
    if (!MMA) return partial_smem_bytes<HD, GM>(HG, mb);
    const size_t q = (size_t)align_up(HG * GM * HD * 4, 128);
    const size_t body = (size_t)NW * MmaWarpArea<HD>::bytes;
    const size_t merge = (size_t)NW * GM * (HD + 2) * 4;
    return q + (body > merge ? body : merge);
}

// MMA: packed chunks run the tensor-core unit (head_dim 64 / 128, GM <= 4, an
// even number of kv heads, fp16 metadata: the host only selects it then);
// otherwise the SIMT unit.  bx = packed chunk of the job.
template <int HD, int GM, bool MMA>
__device__ __forceinline__ void packed_body(const AttnLaunch& L, const JobDesc& J, const TierCounts tc, int bx, int by) {
    constexpr int CPL = HDT<HD>::CPL;
    constexpr int NS = NSTAGE;  // stage slots of SIMT packed chunks
    using WA = WarpArea<HD, GM>;
    extern __shared__ __align__(128) unsigned char smem[];
    __shared__ __align__(8) uint64_t bars[NS];

    const int job = by / L.nhg;
    const int hg = by - job * L.nhg;
    const int D = tc.n0 + tc.n1 + tc.n2;
    // this launch's share of the positions (all of them unless sharded)
    const ShardMap M = shard_map(tc, J.grp, L.rank, L.world);
    const int t0 = bx * L.PC;  // local packed tokens [t0, t1): sharded launches use PC % kShardGran == 0,
    const int t1 = min(M.np, t0 + L.PC);  // so stages and units never cross an ownership granule
    if (t0 >= t1) return;
    const int Dl = M.nd;  // local dense positions precede the local packed ones in the logits

    const int G = L.G, HG = L.HG;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int kvl = warp % HG, r0 = warp / HG, WPH = NW / HG;
    const bool active = warp < HG * WPH;  // with 3, 5, 6 or 7 heads some warps idle
    const int kvh = hg * HG + kvl;
    const float sc = (1.0f / sqrtf((float)HD)) * kLog2e;  // log2-domain logit scale
    const int mb = J.meta16 ? 2 : 4;
    const StageLayout SL = stage_layout(HD, mb, HG);
    const int qbytes = align_up(HG * GM * HD * 4, 128);
    unsigned char* stages = smem + qbytes;
    unsigned char* wa = MMA ? stages + (size_t)warp * MmaWarpArea<HD>::bytes
                            : stages + (size_t)NS * SL.bytes + (size_t)warp * WA::bytes;

    // SIMT packed chunks: start the first bulk copies before staging Q
    const int ST = stage_tokens(HG);
    const int nst = ceil_div(t1 - t0, ST);
    if (!MMA) {
        if (threadIdx.x == 0) {
#pragma unroll
            for (int i = 0; i < NS; ++i) mbar_init(&bars[i], 1);
            mbar_fence_init();
        }
        __syncthreads();
        if (warp == 0)
            for (int s = 0; s < NS && s < nst; ++s)
                pbs_issue_stage<HD, GM>(J, HG, hg, t0, t1, s, stages, SL, bars, lane, L.rank, L.world);
    }

    // ---- query rows of this kv-head group: q_s[kvl][g][c] ----
    float* q_s = reinterpret_cast<float*>(smem);
    const float* __restrict__ Q = L.Q[job];
    for (int i = threadIdx.x; i < HG * GM * HD; i += NT) {
        const int c = i % HD, kg = i / HD, g = kg % GM, kv = kg / GM;
        q_s[i] = g < G ? Q[((size_t)(hg * HG + kv) * G + g) * HD + c] : 0.f;
    }
    __syncthreads();
    const float* qk = q_s + (size_t)kvl * GM * HD;
    // partial slot: this job's active chunks, dense first, packed after (compact,
    // so a job's slots never depend on the other jobs of a batch)
    const int chunk = ceil_div(M.nd, L.DC) + bx;
    float* mbuf = reinterpret_cast<float*>(smem + qbytes);  // merge buffer (aliases the stages / warp areas)

    if (MMA) {
        if constexpr (MMA) {
            // More than 4 query heads per kv head (GM = 8): every kv head is
            // two virtual halves of 4 heads, one warp each (the host then uses
            // kv-head groups of 4, so HGv = 8 and each warp walks all units of
            // the chunk); both halves read the same packed bytes.
            constexpr int GS = GM > 4 ? 2 : 1;
            constexpr int GMv = GM > 4 ? 4 : GM;
            const int HGv = HG * GS;
            const int vw = warp % HGv, r0v = warp / HGv, WPHv = NW / HGv;
            const int kvl_r = vw / GS, half = vw % GS;
            const int kvh_r = hg * HG + kvl_r;
            const int hbase = kvh_r * G + GMv * half;           // first query head of this warp
            const int gcnt = min(GMv, G - GMv * half);         // its query heads
            const bool act = warp < HGv * WPHv && gcnt > 0;
            const float* qv = q_s + (size_t)kvl_r * GM * HD + (size_t)half * GMv * HD;
            MmaState<HD> S;
            S.init();
            MmaQ<HD> Qf;
            // This warp's units: 32-token units r0v, r0v + WPHv, ... of [t0, t1),
            // through its own kMmaSlots-deep cp.async pipeline.
            const int nu_all = ceil_div(t1 - t0, 32);
            const int nu = act && r0v < nu_all ? ceil_div(nu_all - r0v, WPHv) : 0;
            if (nu > 0) {
                mma_prepare_q<HD, GMv>(qv, lane, sc, wa, Qf);
                // the block size is a template parameter of the unit (16 or 32 tokens)
                auto run = [&](auto gsh_tag) {
                    constexpr int GSH = decltype(gsh_tag)::value;
                    auto issue = [&](int k) {
                        const int s0 = t0 + (r0v + k * WPHv) * 32;
                        mma_issue<HD, GSH>(J, kvh_r, packed_global(s0, L.rank, L.world), min(32, t1 - s0),
                                           wa + (size_t)(k % kMmaSlots) * MmaStage<HD>::bytes, lane);
                    };
#pragma unroll
                    for (int k = 0; k < kMmaSlots - 1; ++k) {
                        if (k < nu) issue(k);
                        cp_async_commit();
                    }
                    for (int k = 0; k < nu; ++k) {
                        // refill the slot unit k-1 used (released at the end of its iteration)
                        if (k + kMmaSlots - 1 < nu) issue(k + kMmaSlots - 1);
                        cp_async_commit();
                        cp_async_wait<kMmaSlots - 1>();  // unit k's copies (this lane's) have landed
                        __syncwarp();                    // ... and every lane's are visible
                        const int s0 = t0 + (r0v + k * WPHv) * 32;
                        pbs_unit_mma<HD, GMv, GSH>(J, hbase, gcnt, kvh_r, lane, Dl,
                                                   wa + (size_t)(k % kMmaSlots) * MmaStage<HD>::bytes, s0,
                                                   min(32, t1 - s0), Qf, wa, S);
                    }
                    cp_async_wait<0>();
                };
                if (J.grp == 32) run(std::integral_constant<int, 5>{});
                else run(std::integral_constant<int, 4>{});
            }
            float m, l, o[HD / 16][2];
            mma_finish<HD>(S, m, l, o);
            const int gid = lane >> 2, tig = lane & 3;
            if (WPHv == 1) {
                if (!act || tig >= gcnt) return;
                const size_t pi = (size_t)chunk * J.nq + hbase + tig;
                if (gid == 0) {
                    J.part_ml[pi * 2 + 0] = m;
                    J.part_ml[pi * 2 + 1] = l;
                }
#pragma unroll
                for (int mt = 0; mt < HD / 16; ++mt) {
                    J.part_acc[pi * HD + 16 * mt + gid] = o[mt][0];
                    J.part_acc[pi * HD + 16 * mt + gid + 8] = o[mt][1];
                }
                return;
            }
            if constexpr (GS == 1) {  // several warps per kv head: merge them
                __syncthreads();
                if (active && tig < GM) {
                    float* mine = mbuf + (size_t)warp * GM * (HD + 2) + tig * (HD + 2);
                    if (gid == 0) {
                        mine[0] = m;
                        mine[1] = l;
                    }
#pragma unroll
                    for (int mt = 0; mt < HD / 16; ++mt) {
                        mine[2 + 16 * mt + gid] = o[mt][0];
                        mine[2 + 16 * mt + gid + 8] = o[mt][1];
                    }
                }
                __syncthreads();
                if (r0 != 0 || !active) return;
                merge_warps<HD, GM>(J, mbuf, chunk, kvh, kvl, HG, WPH, G, lane);
            }
        }
        return;
    }

    WarpState<HD, GM> S;
    S.init();
    bool failed = false;
    {
        int s = 0;
        for (; s < nst; ++s) {
            const bool ok = mbar_wait_bounded(&bars[s % NSTAGE], (uint32_t)((s / NSTAGE) & 1));
            if (__syncthreads_or(!ok)) {
                failed = true;
                break;
            }
            const unsigned char* buf = stages + (size_t)(s % NSTAGE) * SL.bytes;
            const int s0 = t0 + s * ST;
            const int nt = min(ST, t1 - s0);
            if (active && r0 * 32 < nt) pbs_unit<HD, GM>(J, HG, G, kvl, kvh, lane, Dl, buf, SL, s0, nt, r0, qk, wa, sc, S);
            __syncthreads();
            if (warp == 0 && s + NSTAGE < nst) pbs_issue_stage<HD, GM>(J, HG, hg, t0, t1, s + NSTAGE, stages, SL, bars, lane, L.rank, L.world);
        }
        if (failed) {
            // drain this CTA's own copies in flight, then give up on the chunk
            for (int k = s; k < nst && k < s + NSTAGE; ++k)
                (void)mbar_wait_bounded(&bars[k % NSTAGE], (uint32_t)((k / NSTAGE) & 1));
            if (threadIdx.x == 0) {
                atomicCAS(&g_device_error, 0, (int)TT_ERR_TIMEOUT);
                if (J.ctr) atomicCAS(const_cast<int*>(&J.ctr->error), 0, (int)TT_ERR_TIMEOUT);
            }
            return;
        }
    }

    // ---- per-warp totals ----
    float out[GM][CPL];
#pragma unroll
    for (int g = 0; g < GM; ++g) {
        S.l[g] = warp_sum(S.l[g]);
        const float SW = warp_sum(S.sws[g]);
        const float SZ = warp_sum(S.spz[g]);
        if constexpr (CPL >= 2) {
#pragma unroll
            for (int q = 0; q < CPL / 2; ++q) {
                const float2 v = f2unpack(S.acc2[g][q]);
                out[g][2 * q] = v.x;
                out[g][2 * q + 1] = v.y;
            }
        } else {
            out[g][0] = S.acc1[g];
        }
#pragma unroll
        for (int j = 0; j < CPL; ++j) out[g][j] = (out[g][j] - 4.0f * SW) + SZ;
    }

    if (WPH == 1) {
        if (!active) return;
#pragma unroll
        for (int g = 0; g < GM; ++g) {
            if (g >= G) break;
            const size_t pi = part_index(J, chunk, kvh, G, g);
            if (lane == 0) {
                J.part_ml[pi * 2 + 0] = S.m[g];
                J.part_ml[pi * 2 + 1] = S.l[g];
            }
#pragma unroll
            for (int j = 0; j < CPL; ++j) {
                const int c = lane * CPL + j;
                if (c < HD) J.part_acc[pi * HD + c] = out[g][j];
            }
        }
        return;
    }
    // ---- merge the WPH warps that share a kv head (buffer aliases the stages) ----
    __syncthreads();
    float* mine = mbuf + (size_t)warp * GM * (HD + 2);
#pragma unroll
    for (int g = 0; g < GM; ++g) {
        if (lane == 0) {
            mine[g * (HD + 2) + 0] = S.m[g];
            mine[g * (HD + 2) + 1] = S.l[g];
        }
#pragma unroll
        for (int j = 0; j < CPL; ++j) {
            const int c = lane * CPL + j;
            if (c < HD) mine[g * (HD + 2) + 2 + c] = out[g][j];
        }
    }
    __syncthreads();
    if (r0 != 0 || !active) return;
    merge_warps<HD, GM>(J, mbuf, chunk, kvh, kvl, HG, WPH, G, lane);
}

// Arrival counter of a job's chunk CTAs: the partials' spare chunk slot
// max_chunks - 2 (a job's active chunks use at most max_chunks - 2 slots).
// Zero between launches: the engine clears its scratch when it (re)sizes it
// and the merging CTA resets the counter.
__device__ __forceinline__ int* job_counter(const JobDesc& J) {
    return reinterpret_cast<int*>(J.part_ml + (size_t)(J.max_chunks - 2) * J.nq * 2);
}

// After the CTA's own chunk: the last CTA of its job merges the job's chunk
// partials per head -- M = max m, L = sum l 2^(m - M), acc = sum acc 2^(m - M)
// (row_sum_exp fallback, fused_attn_avx2.cpp:261) -- into attn_output and
// (M, 1/L) (merge_mode 1, what k_attn_merge_heads computes) or into the job's
// exchange row (merge_mode 2, what k_shard_local_merge computes).  TPH threads
// per head, each owning float4 channel groups, with many chunks' loads in
// flight.  Release / acquire as in a grid barrier: CTA barrier, then one
// thread fences and arrives; the merging CTA fences after the last arrival and
// reads the partials through L2.
template <int HD>
__device__ __forceinline__ void chunk_merge_tail(const AttnLaunch& L, const JobDesc& J, const TierCounts tc, int job) {
    constexpr int TPH = HD >= 32 ? 8 : 4;      // threads per head
    constexpr int V4 = HD / (4 * TPH);         // float4 groups per thread (channels 4 (tq + TPH v) ..)
    constexpr int HPP = NT / TPH;              // heads per pass
    __shared__ int last;
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence();
        last = atomicAdd(job_counter(J), 1) == (L.nd + L.np) * L.nhg - 1;
        if (last) __threadfence();
    }
    __syncthreads();
    if (!last) return;
    const int nq = J.nq;
    const ShardMap M = shard_map(tc, J.grp, L.rank, L.world);
    const int nch = ceil_div(M.nd, L.DC) + ceil_div(M.np, L.PC);
    const int tq = threadIdx.x % TPH;
    const float2* pml = reinterpret_cast<const float2*>(J.part_ml);
    for (int h = threadIdx.x / TPH; h < nq; h += HPP) {  // the TPH threads of a head are adjacent lanes
        float M = -INFINITY;
        for (int i = tq; i < nch; i += TPH) M = fmaxf(M, __ldcg(&pml[(size_t)i * nq + h].x));
#pragma unroll
        for (int x = 1; x < TPH; x <<= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, x));
        float S = 0.f;
        float4 o[V4];
#pragma unroll
        for (int v = 0; v < V4; ++v) o[v] = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll 8
        for (int i = 0; i < nch; ++i) {
            const float2 p = __ldcg(&pml[(size_t)i * nq + h]);
            const float w = (M == -INFINITY || p.x == -INFINITY) ? 0.f : exp2f(p.x - M);
            S = fmaf(p.y, w, S);
            const float4* a = reinterpret_cast<const float4*>(J.part_acc + ((size_t)i * nq + h) * HD) + tq;
#pragma unroll
            for (int v = 0; v < V4; ++v) {
                const float4 x = __ldcg(a + TPH * v);
                o[v].x = fmaf(x.x, w, o[v].x);
                o[v].y = fmaf(x.y, w, o[v].y);
                o[v].z = fmaf(x.z, w, o[v].z);
                o[v].w = fmaf(x.w, w, o[v].w);
            }
        }
        if (L.merge_mode == 2) {
            // the job's row: into the exchange buffer, or into every rank's
            // region (peer memory over NVLink) at this rank's slot
            const int nw = L.px.world > 1 ? L.px.world : 1;
            for (int p = 0; p < nw; ++p) {
                float* xr = L.px.world > 1
                                ? L.px.rows[p] + (((size_t)L.px.rank * L.px.jobs + job) * nq + h) * (HD + 2)
                                : L.xch + ((size_t)job * nq + h) * (HD + 2);
#pragma unroll
                for (int v = 0; v < V4; ++v) {
                    const int c = 4 * (tq + TPH * v);
                    xr[2 + c] = o[v].x;
                    xr[3 + c] = o[v].y;
                    xr[4 + c] = o[v].z;
                    xr[5 + c] = o[v].w;
                }
                if (tq == 0) {
                    xr[0] = M;
                    xr[1] = S;
                }
            }
            if (threadIdx.x == 0 && h == 0) *route_min_word(J) = 0ull;
        } else {
            const float inv = 1.0f / (S > 0.f ? S : 1.0f);
            float* out = L.out[job] + (size_t)h * HD;
            if ((reinterpret_cast<uintptr_t>(L.out[job]) & 15) == 0) {
#pragma unroll
                for (int v = 0; v < V4; ++v)
                    reinterpret_cast<float4*>(out)[tq + TPH * v] =
                        make_float4(o[v].x * inv, o[v].y * inv, o[v].z * inv, o[v].w * inv);
            } else {  // attn_output need not be 16-byte aligned
#pragma unroll
                for (int v = 0; v < V4; ++v) {
                    const int c = 4 * (tq + TPH * v);
                    out[c] = o[v].x * inv;
                    out[c + 1] = o[v].y * inv;
                    out[c + 2] = o[v].z * inv;
                    out[c + 3] = o[v].w * inv;
                }
            }
            if (tq == 0) {
                float* ml = head_ml(J);  // (M, 1/L) for the weights pass
                ml[2 * h] = M;
                ml[2 * h + 1] = inv;
            }
        }
    }
    if (L.merge_mode == 2 && L.px.world > 1) {
        __syncthreads();  // every thread's row stores are issued before the flags
        if (threadIdx.x == 0) {
            __threadfence_system();
            for (int p = 0; p < L.px.world; ++p)
                st_release_sys(L.px.flags[p] + (size_t)L.px.rank * L.px.jobs + job, (unsigned long long)L.px.step);
        }
    }
    if (threadIdx.x == 0) *job_counter(J) = 0;
}

// grid (np, njobs * nhg).  With merge_mode set, the job's last CTA (of this
// kernel or of the dense one) merges the job's chunks (chunk_merge_tail);
// every CTA arrives, also those without tokens.
template <int HD, int GM, bool MMA>
__global__ void __launch_bounds__(NT, (GM >= 8 && !MMA) ? 1 : 2) k_attn_packed(const __grid_constant__ AttnLaunch L) {
    __shared__ JobDesc Js;
    __shared__ TierCounts Ts;
    const int job = blockIdx.y / L.nhg;
    if (threadIdx.x == 0) {
        Js = L.jobs[job] ? *L.jobs[job] : L.inline_job;
        Ts = resolve_counts(Js);
    }
    __syncthreads();
    packed_body<HD, GM, MMA>(L, Js, Ts, blockIdx.x, blockIdx.y);
    if (L.merge_mode) chunk_merge_tail<HD>(L, Js, Ts, job);
}

}  // namespace tt
