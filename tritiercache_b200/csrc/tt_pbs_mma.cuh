// tt_pbs_mma.cuh -- packed-tier (2-bit) attention on the tensor cores with
// mma.sync.m16n8k16 (f16 operands, f32 accumulation).  Included by
// tt_partial.cuh.  Used for head_dim 64 / 128, at most 4 query heads per kv
// head, an even number of kv heads and fp16 metadata; the SIMT unit covers the
// other shapes.
//
// Fragment layout of m16n8k16 (row.col); lane = 4*gid + tig:
//   A a0:(row gid, k-slots 2tig,2tig+1) a1:(gid+8, same) a2:(gid, 2tig+8,+9) a3:(gid+8, same)
//   B b0:(k-slots 2tig,2tig+1; n=gid)   b1:(k-slots 2tig+8,+9; n=gid)
//   D d0,d1:(row gid, n=2tig,2tig+1)    d2,d3:(row gid+8, same)
// Any k-slot <-> element permutation works as long as A and B use the same
// one: k-slots (2tig, 2tig+1, 2tig+8, 2tig+9) map to channels 16ks+4tig+{0..3}
// in QK (one 16-byte load of K words, one 8-byte load of scales) and to tokens
// tig+4i (i = 0..3) of a 16-token step in PV (bank-conflict-free V loads).
//
// Columns n = 2g + part: head g, part 0 = f16 "hi", part 1 = f16 "lo" of the
// same f32 operand, so one f32 accumulation carries ~22 significant bits.
//
// QK per 16-token half-unit, score[t][g] = sum_c (q_c s_c) (4 + code_tc):
//   A = 4 + code as f16 (exact): the 2-bit fields of rows gid and gid+8 sit in
//       bytes gid/4 and 2+gid/4 of each K word (16 tokens of one channel);
//       one PRMT gathers them from two words, a shift + LOP3 each places them
//       in the mantissa of f16 4.0.
//   B = q' * s split into hi/lo with f16 FMAs: h = q'h*s, r = q'h*s - h (exact),
//       lo = q'l*s + r; q' = q * 2^-e_g with |q'| < 1, so |q' s| <= 65504.
//   bias = -4 sum_c q' s + sum_c q' z: one MMA per k-step with the scale rows
//       (A rows 0..7) and zero rows (8..15) of both blocks and the q' fragments as B.
// PV per 32-token unit, out[c][g] = sum_t (p_t vs_t) (4 + code_tc):
//   A = 4 + code from the V words (16 channels of one token), same gather;
//   B = p*vs*2^-E split hi/lo; E is kept while a unit's largest weight stays
//   in [2^4, 2^14) * 2^E (else reset to put it near 2^13).  Each unit's
//   tile result (hi + lo columns) is folded into the running f32 output as
//   acc = acc * alpha * 2^(E_old - E_new) + tile.
// In both D layouts a thread holds query head g = tig.
//
// Staging: each warp runs its own two-slot pipeline over its units.  Its part
// of a unit (K words, block scales/zeros, V words, V scale/zero, ids: 3.5 KB
// at head_dim 128) moves with per-lane 16-byte cp.async (4-byte for the V
// scale/zero pairs) into a warp-private slot, waited for with
// cp.async.wait_group + __syncwarp.  No warp waits for another, and no copy is
// small enough to be issue-bound.
#pragma once

namespace tt {

constexpr int kMmaWRow = 48;   // halves per row of the PV weight table (32 tokens + pad)
constexpr int kMmaSlots = 2;   // stages in flight per warp

// One warp's stage: its kv head's part of one 32-token unit.
template <int HD>
struct MmaStage {
    static constexpr int kw = 0;                   // [2 rows of 16 tokens][HD] K words
    static constexpr int ks = kw + 2 * HD * 4;     // [2 blocks][HD] f16 K scales (1 block used with group 32)
    static constexpr int kz = ks + 2 * HD * 2;     // [2 blocks][HD] f16 K zeros
    static constexpr int vw = kz + 2 * HD * 2;     // [32 tokens][HD/16] V words
    static constexpr int vs = vw + 32 * HD / 4;    // [32 tokens][2] f16 V scales of heads (h & ~1, h | 1)
    static constexpr int vz = vs + 32 * 4;         // same for the V zeros
    static constexpr int ids = vz + 32 * 4;        // [32] token ids
    static constexpr int bytes = (ids + 32 * 8 + 127) / 128 * 128;
};

// Per-warp shared memory of the tensor-core unit: its stage slots, the PV
// weight table and the q' hi table.
template <int HD>
struct MmaWarpArea {
    static constexpr int slots = kMmaSlots * MmaStage<HD>::bytes;
    static constexpr int wtab = slots;                  // [n][position] f16
    static constexpr int qtab = wtab + 8 * kMmaWRow * 2; // [ks][head*4 + tig | 16 + tig][2] f16x2: q' hi | zero
    static constexpr int bytes = (qtab + (HD / 16) * 40 * 4 + 127) / 128 * 128;
};

__device__ __forceinline__ void mma_f16_16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                              uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t h2u(__half2 h) { return *reinterpret_cast<uint32_t*>(&h); }
__device__ __forceinline__ __half2 u2h(uint32_t u) { return *reinterpret_cast<__half2*>(&u); }
__device__ __forceinline__ float pow2f(int e) { return __uint_as_float((uint32_t)(127 + e) << 23); }  // |e| <= 126

// cp.async of 4 bytes (L1-allocating form; the 16-byte form is cp_async16)
__device__ __forceinline__ void cp_async4(void* dst, const void* src) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_addr(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// d += A*B (ZERO_C: d = A*B) where A is the 4+code fragment of the k-slot
// pairs (w0, w1) and (w2, w3) for rows gid and gid+8: sel gathers byte gid/4
// and 2+gid/4 of both words (PRMT), the fields move to mantissa bits 8-9 of
// each f16 half by a multiply with m8 = 2^(8 - sft) (row gid, on the FMA pipe)
// or a right shift by sft = 2*(gid%4) (row gid+8), and LOP3 masks them and
// sets the exponent of 4.0.  One PTX block, so the LOP3 results are the MMA's
// operand registers.
template <bool ZERO_C>
__device__ __forceinline__ void mma_codes(float (&d)[4], uint32_t w0, uint32_t w1, uint32_t w2, uint32_t w3,
                                          uint32_t sel, uint32_t sft, uint32_t m8, uint32_t b0, uint32_t b1) {
    if constexpr (ZERO_C) {
        asm volatile(
            "{\n .reg .b32 p0, p1, t0, t1, t2, t3, a0, a1, a2, a3;\n"
            " prmt.b32 p0, %4, %5, %8;\n prmt.b32 p1, %6, %7, %8;\n"
            " mul.lo.u32 t0, p0, %10;\n shr.b32 t1, p0, %9;\n mul.lo.u32 t2, p1, %10;\n shr.b32 t3, p1, %9;\n"
            " lop3.b32 a0, t0, 0x03000300, 0x44004400, 0xea;\n lop3.b32 a1, t1, 0x03000300, 0x44004400, 0xea;\n"
            " lop3.b32 a2, t2, 0x03000300, 0x44004400, 0xea;\n lop3.b32 a3, t3, 0x03000300, 0x44004400, 0xea;\n"
            " mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {a0,a1,a2,a3}, {%11,%12}, "
            "{%13,%13,%13,%13};\n}\n"
            : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
            : "r"(w0), "r"(w1), "r"(w2), "r"(w3), "r"(sel), "r"(sft), "r"(m8), "r"(b0), "r"(b1), "f"(0.f));
    } else {
        asm volatile(
            "{\n .reg .b32 p0, p1, t0, t1, t2, t3, a0, a1, a2, a3;\n"
            " prmt.b32 p0, %4, %5, %8;\n prmt.b32 p1, %6, %7, %8;\n"
            " mul.lo.u32 t0, p0, %10;\n shr.b32 t1, p0, %9;\n mul.lo.u32 t2, p1, %10;\n shr.b32 t3, p1, %9;\n"
            " lop3.b32 a0, t0, 0x03000300, 0x44004400, 0xea;\n lop3.b32 a1, t1, 0x03000300, 0x44004400, 0xea;\n"
            " lop3.b32 a2, t2, 0x03000300, 0x44004400, 0xea;\n lop3.b32 a3, t3, 0x03000300, 0x44004400, 0xea;\n"
            " mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {a0,a1,a2,a3}, {%11,%12}, "
            "{%0,%1,%2,%3};\n}\n"
            : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
            : "r"(w0), "r"(w1), "r"(w2), "r"(w3), "r"(sel), "r"(sft), "r"(m8), "r"(b0), "r"(b1));
    }
}

// B register (n = gid) of q'*s for two channels.  qm is q' hi on lo (odd)
// lanes and zero on hi (even) lanes, qx the lane's own part of q': hi lanes
// get round(q'h*s), lo lanes q'l*s + (q'h*s - round(q'h*s)), the residual
// being exact in f16.
__device__ __forceinline__ uint32_t b_qs(uint32_t qm, uint32_t qx, uint32_t s) {
    const __half2 sv = u2h(s), qmv = u2h(qm);
    const __half2 h = __hmul2(qmv, sv);
    const __half2 r = __hfma2(qmv, sv, __hneg2(h));
    return h2u(__hfma2(u2h(qx), sv, r));
}

// Per-thread B fragments of q' for n = gid (head gid/2, part gid&1) and the
// power-of-two scale of head tig.  The hi part, which the lo lanes also need,
// goes to the warp's q table (with zero rows that the hi lanes read).
template <int HD>
struct MmaQ {
    static constexpr int KS = HD / 16;
    uint32_t qx[KS][2];  // the B fragment of q' itself: hi (even gid) or lo (odd gid)
    float up_sc;         // 2^e of head tig times the log2-domain logit scale
};

template <int HD, int GM>
__device__ __forceinline__ void mma_prepare_q(const float* qk, int lane, float sc, unsigned char* wa, MmaQ<HD>& Q) {
    constexpr int KS = HD / 16;
    const int gid = lane >> 2, tig = lane & 3;
    const int g = gid >> 1;
    float4 v[KS];
    float mx = 0.f;
#pragma unroll
    for (int ks = 0; ks < KS; ++ks) {
        v[ks] = g < GM ? *reinterpret_cast<const float4*>(qk + g * HD + 16 * ks + 4 * tig) : make_float4(0.f, 0.f, 0.f, 0.f);
        mx = fmaxf(mx, fmaxf(fmaxf(fabsf(v[ks].x), fabsf(v[ks].y)), fmaxf(fabsf(v[ks].z), fabsf(v[ks].w))));
    }
    // lanes of one head differ in tig (xor 1, 2) and part (xor 4)
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 4));
    // e with mx * 2^-e in [0.5, 1); zero rows keep e = 0
    int e = mx > 0.f ? (int)((__float_as_uint(mx) >> 23) & 0xff) - 126 : 0;
    e = max(-100, min(100, e));
    const float down = pow2f(-e);
    const bool odd = (gid & 1) != 0;
    uint32_t* qtab = reinterpret_cast<uint32_t*>(wa + MmaWarpArea<HD>::qtab);
#pragma unroll
    for (int ks = 0; ks < KS; ++ks) {
        const float x0 = v[ks].x * down, x1 = v[ks].y * down, x2 = v[ks].z * down, x3 = v[ks].w * down;
        const __half2 h01 = __floats2half2_rn(x0, x1), h23 = __floats2half2_rn(x2, x3);
        const float2 f01 = __half22float2(h01), f23 = __half22float2(h23);
        const __half2 l01 = __floats2half2_rn(x0 - f01.x, x1 - f01.y), l23 = __floats2half2_rn(x2 - f23.x, x3 - f23.y);
        if (!odd) *reinterpret_cast<uint2*>(qtab + ks * 40 + (g * 4 + tig) * 2) = make_uint2(h2u(h01), h2u(h23));
        if (gid == 0) *reinterpret_cast<uint2*>(qtab + ks * 40 + (16 + tig) * 2) = make_uint2(0u, 0u);
        Q.qx[ks][0] = odd ? h2u(l01) : h2u(h01);
        Q.qx[ks][1] = odd ? h2u(l23) : h2u(h23);
    }
    // head tig's exponent lives on lane 8*tig (gid = 2*tig)
    const int et = __shfl_sync(0xffffffffu, e, 8 * tig);
    Q.up_sc = pow2f(et) * sc;
    __syncwarp();
}

template <int HD>
struct MmaState {
    static constexpr int MT = HD / 16;
    float m, l, sws, spz;  // head tig; l / sws / spz over this thread's tokens only
    int E;                 // exponent of the PV accumulator
    float acc[MT][2];      // channels 16mt+gid and 16mt+gid+8 (hi + lo columns folded)
    __device__ __forceinline__ void init() {
        m = -INFINITY; l = 0.f; sws = 0.f; spz = 0.f; E = 0;
#pragma unroll
        for (int i = 0; i < MT; ++i) { acc[i][0] = 0.f; acc[i][1] = 0.f; }
    }
};

// Copies the warp's part of the unit [s0, s0 + nt) (nt = 16 or 32) for kv head
// kvh into stage st with per-lane cp.async; the caller commits the group.
// Every source offset is a multiple of 16 bytes (4 for the V scale/zero pairs:
// the number of kv heads is even), every size a multiple of the copy size.
template <int HD, int GSH>
__device__ __forceinline__ void mma_issue(const JobDesc& J, int kvh, int s0, int nt, unsigned char* st, int lane) {
    using SL = MmaStage<HD>;
    constexpr int DQ = HD / 16;
    const int nkv = J.nkv;
    constexpr int gsh = GSH;  // log2 of the block size (16 or 32)
    // per-array bases of this unit (uniform across the warp) + 32-bit lane offsets
    const char* kb = reinterpret_cast<const char*>(J.kp) + ((size_t)(s0 >> 4) * nkv + kvh) * (HD * 4);
    const size_t moff = ((size_t)(s0 >> gsh) * nkv + kvh) * (HD * 2);
    const char* sb = reinterpret_cast<const char*>(J.ks) + moff;
    const char* zb = reinterpret_cast<const char*>(J.kz) + moff;
    const char* vb = reinterpret_cast<const char*>(J.vp) + ((size_t)s0 * nkv + kvh) * (DQ * 4);
    const size_t soff = ((size_t)s0 * nkv + (kvh & ~1)) * 2;
    const char* vsb = reinterpret_cast<const char*>(J.vs) + soff;
    const char* vzb = reinterpret_cast<const char*>(J.vz) + soff;
    const char* ib = reinterpret_cast<const char*>(J.ids) + (size_t)s0 * 8;
    const int krow = nkv * HD * 4;            // bytes between K word rows (16 tokens)
    const int mblk = nkv * HD * 2;            // bytes between metadata blocks
    const int vtok = nkv * DQ * 4;            // bytes between tokens' V words
    if (nt == 32) {
        // a full unit: every lane's pieces are fixed (straight-line issue)
#pragma unroll
        for (int j = 0; j < HD / 64; ++j) {  // K words: 2 rows x HD/4 chunks
            const int i = lane + 32 * j, r = i / (HD / 4), c = i % (HD / 4);
            cp_async16(st + SL::kw + r * HD * 4 + c * 16, kb + r * krow + c * 16);
        }
        if (gsh == 4 || lane < HD / 8) {  // K scale / zero: (32 >> gsh) blocks x HD/8 chunks
            const int b = lane / (HD / 8), c = lane % (HD / 8);
            if (HD == 64) {  // 8 chunks per block: lanes 0..15 cover both blocks
                if (lane < (32 >> gsh) * (HD / 8)) {
                    cp_async16(st + SL::ks + b * HD * 2 + c * 16, sb + b * mblk + c * 16);
                    cp_async16(st + SL::kz + b * HD * 2 + c * 16, zb + b * mblk + c * 16);
                }
            } else {
                cp_async16(st + SL::ks + b * HD * 2 + c * 16, sb + b * mblk + c * 16);
                cp_async16(st + SL::kz + b * HD * 2 + c * 16, zb + b * mblk + c * 16);
            }
        }
#pragma unroll
        for (int j = 0; j < HD / 64; ++j) {  // V words: 32 tokens x HD/64 chunks
            const int i = lane + 32 * j, t = i / (HD / 64), c = i % (HD / 64);
            cp_async16(st + SL::vw + t * DQ * 4 + c * 16, vb + t * vtok + c * 16);
        }
        cp_async4(st + SL::vs + lane * 4, vsb + lane * nkv * 2);
        cp_async4(st + SL::vz + lane * 4, vzb + lane * nkv * 2);
        if (lane < 16) cp_async16(st + SL::ids + lane * 16, ib + lane * 16);
        return;
    }
    const int rows = nt >> 4;
    for (int i = lane; i < rows * (HD / 4); i += 32) {  // K words: HD/4 chunks per row
        const int r = i / (HD / 4), c = i % (HD / 4);
        cp_async16(st + SL::kw + r * HD * 4 + c * 16, kb + r * krow + c * 16);
    }
    const int nb = max(1, nt >> gsh);
    for (int i = lane; i < nb * (HD / 8); i += 32) {  // K scale / zero: HD/8 chunks per block
        const int b = i / (HD / 8), c = i % (HD / 8);
        cp_async16(st + SL::ks + b * HD * 2 + c * 16, sb + b * mblk + c * 16);
        cp_async16(st + SL::kz + b * HD * 2 + c * 16, zb + b * mblk + c * 16);
    }
    for (int i = lane; i < nt * (HD / 64); i += 32) {  // V words: HD/64 chunks per token
        const int t = i / (HD / 64), c = i % (HD / 64);
        cp_async16(st + SL::vw + t * DQ * 4 + c * 16, vb + t * vtok + c * 16);
    }
    if (lane < nt) {  // V scale / zero of heads (kvh & ~1, kvh | 1)
        cp_async4(st + SL::vs + lane * 4, vsb + lane * nkv * 2);
        cp_async4(st + SL::vz + lane * 4, vzb + lane * nkv * 2);
    }
    if (lane < nt / 2) cp_async16(st + SL::ids + lane * 16, ib + lane * 16);
}

// position of unit-local token t in the PV weight table (k-slot order)
__device__ __forceinline__ int mma_wpos(int t) { return (t & 16) + 4 * (t & 3) + ((t & 15) >> 2); }

__device__ __forceinline__ float ex2_approx(float x) {  // 2^x (PTX ex2.approx; -inf -> +0)
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// One 32-token unit [s0, s0 + nt) of kv head kvh from stage st.
template <int HD, int GM, int GSH>
// hbase / gcnt: the first of this warp's query heads and how many there are
// (<= 4); kvh: the kv head whose packed bytes the unit reads; GSH: log2 of the
// block size (4: 16 tokens, 5: 32 tokens).
__device__ __forceinline__ void pbs_unit_mma(const JobDesc& J, int hbase, int gcnt, int kvh, int lane, int D,
                                             const unsigned char* st, int s0, int nt, const MmaQ<HD>& Q,
                                             unsigned char* wa, MmaState<HD>& S) {
    static_assert((HD == 64 || HD == 128) && GM <= 4, "tensor-core unit shape");
    using SL = MmaStage<HD>;
    constexpr int KS = HD / 16, DQ = HD / 16;
    const int gid = lane >> 2, tig = lane & 3;
    const uint32_t sft = 2 * (gid & 3);
    const uint32_t m8 = 1u << (8 - sft);
    const uint32_t sel = 0x6420u + 0x1111u * (uint32_t)(gid >> 2);
    __half* wtab = reinterpret_cast<__half*>(wa + MmaWarpArea<HD>::wtab);
    constexpr int gsh = GSH;
    const uint32_t* kw_s = reinterpret_cast<const uint32_t*>(st + SL::kw);
    const __half* ks_s = reinterpret_cast<const __half*>(st + SL::ks);
    const __half* kz_s = reinterpret_cast<const __half*>(st + SL::kz);
    const uint32_t* vw_s = reinterpret_cast<const uint32_t*>(st + SL::vw);
    const __half* vs_s = reinterpret_cast<const __half*>(st + SL::vs) + (kvh & 1);
    const __half* vz_s = reinterpret_cast<const __half*>(st + SL::vz) + (kvh & 1);
    const int64_t* ids_s = reinterpret_cast<const int64_t*>(st + SL::ids);
    // Second half-unit present?  (nt is 16 or 32.)  When it is not, its rows
    // still run through the MMAs on whatever the slot holds (in bounds); every
    // value derived from them is masked.
    const bool two = nt > 16;

    // ---- bias rows and QK, three independent accumulation chains ----
    // bias A rows: row gid = scale, row gid+8 = zero of the block of half gid&1
    // (lanes 0..7 carry the two halves; the other rows repeat them, unused)
    float bd[4] = {0.f, 0.f, 0.f, 0.f};
    float dq[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
    {
        // the bias rows' scales are the B fragments' scales of block gid&1
        // (sv0 / sv1 below); their zeros come with one 8-byte load
        const int mo = ((16 * (gid & 1)) >> gsh) * HD + 4 * tig;
        const __half* mz_row = kz_s + mo;
        constexpr bool shared_blk = gsh == 5;  // both halves in one block: same B fragments
        const uint32_t* kw0 = kw_s + 4 * tig;
        const uint32_t* kw1 = kw0 + HD;
        const __half* sb0 = ks_s + 4 * tig;
        const __half* sb1 = ks_s + (16 >> gsh) * HD + 4 * tig;
        // bias rows of half gid&1: that block's scales (one more 8-byte load per
        // k-step instead of two selects)
        const __half* sbb = (!shared_blk && (gid & 1)) ? sb1 : sb0;
        const uint32_t* qm_t = reinterpret_cast<const uint32_t*>(wa + MmaWarpArea<HD>::qtab) +
                               ((gid & 1) ? (gid >> 1) * 4 + tig : 16 + tig) * 2;
#pragma unroll
        for (int ks = 0; ks < KS; ++ks) {
            const uint4 w0 = *reinterpret_cast<const uint4*>(kw0 + 16 * ks);
            const uint4 w1 = *reinterpret_cast<const uint4*>(kw1 + 16 * ks);
            const uint2 sv0 = *reinterpret_cast<const uint2*>(sb0 + 16 * ks);
            const uint2 zv = *reinterpret_cast<const uint2*>(mz_row + 16 * ks);
            const uint2 qm = *reinterpret_cast<const uint2*>(qm_t + ks * 40);
            uint2 sv1 = sv0;
            if constexpr (!shared_blk) sv1 = *reinterpret_cast<const uint2*>(sb1 + 16 * ks);
            const uint2 svb = *reinterpret_cast<const uint2*>(sbb + 16 * ks);
            mma_f16_16816(bd, svb.x, zv.x, svb.y, zv.y, Q.qx[ks][0], Q.qx[ks][1]);
            const uint32_t b00 = b_qs(qm.x, Q.qx[ks][0], sv0.x);
            const uint32_t b01 = b_qs(qm.y, Q.qx[ks][1], sv0.y);
            uint32_t b10 = b00, b11 = b01;
            if constexpr (!shared_blk) {
                b10 = b_qs(qm.x, Q.qx[ks][0], sv1.x);
                b11 = b_qs(qm.y, Q.qx[ks][1], sv1.y);
            }
            mma_codes<false>(dq[0], w0.x, w0.y, w0.z, w0.w, sel, sft, m8, b00, b01);
            mma_codes<false>(dq[1], w1.x, w1.y, w1.z, w1.w, sel, sft, m8, b10, b11);
        }
    }
    // this lane's half (gid&1), head tig: sum q'z - 4 sum q's
    const float bias_own = (bd[2] + bd[3]) - 4.0f * (bd[0] + bd[1]);
    float s[4];  // unit-local tokens gid, gid+8, 16+gid, 24+gid; head tig
    // live tokens of the unit (present and not tombstoned): one id per lane
    const uint32_t live_mask = __ballot_sync(0xffffffffu, lane < nt && ids_s[lane] != -1);
#pragma unroll
    for (int hf = 0; hf < 2; ++hf) {
        const float bias = __shfl_sync(0xffffffffu, bias_own, 4 * hf + tig);
#pragma unroll
        for (int j = 0; j < 2; ++j) {
            const int t = 16 * hf + gid + 8 * j;
            const bool live = tig < gcnt && ((live_mask >> t) & 1u);
            s[2 * hf + j] = live ? ((dq[hf][2 * j] + dq[hf][2 * j + 1]) + bias) * Q.up_sc : -INFINITY;
        }
    }
    // ---- logits to scratch ----
    if (tig < gcnt) {
        float* srow = J.scores + (size_t)(hbase + tig) * J.score_stride + D + s0;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const int t = 16 * (k >> 1) + gid + 8 * (k & 1);
            if (k < 2 || two) st_logit(srow + t, s[k]);
        }
    }
    // ---- online softmax for head tig ----
    float mu = fmaxf(fmaxf(s[0], s[1]), fmaxf(s[2], s[3]));
    mu = fmaxf(mu, __shfl_xor_sync(0xffffffffu, mu, 4));
    mu = fmaxf(mu, __shfl_xor_sync(0xffffffffu, mu, 8));
    mu = fmaxf(mu, __shfl_xor_sync(0xffffffffu, mu, 16));
    const float mn = fmaxf(S.m, mu);
    float alpha = 1.f;
    float p[4] = {0.f, 0.f, 0.f, 0.f};
    if (mn != -INFINITY) {
        alpha = ex2_approx(S.m - mn);
#pragma unroll
        for (int k = 0; k < 4; ++k) p[k] = ex2_approx(s[k] - mn);
    }
    S.m = mn;
    S.l = fmaf(S.l, alpha, (p[0] + p[1]) + (p[2] + p[3]));
    S.sws *= alpha;
    S.spz *= alpha;
    // ---- PV weights p*vs: running sums, accumulator exponent, hi/lo table ----
    float ws[4];
    float wmx = 0.f;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        const int t = 16 * (k >> 1) + gid + 8 * (k & 1);
        float vsc = 0.f, vzr = 0.f;
        if (k < 2 || two) {
            vsc = __half2float(vs_s[2 * t]);
            vzr = __half2float(vz_s[2 * t]);
        }
        ws[k] = p[k] * vsc;
        S.sws += ws[k];
        S.spz = fmaf(p[k], vzr, S.spz);
        wmx = fmaxf(wmx, fabsf(ws[k]));
    }
    // keep the exponent unless the unit's largest weight leaves [2^4, 2^14) * 2^E
    const uint32_t wmb = __reduce_max_sync(0xffffffffu, __float_as_uint(wmx));
    const int we = (int)((wmb >> 23) & 0xff) - 127;
    int En = S.E;
    if (wmb != 0u && (we - S.E >= 14 || we - S.E < 4)) En = max(-40, min(40, we - 13));
    const float f = alpha * pow2f(S.E - En);
    S.E = En;
    const float down = pow2f(-En);
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        const int tl = 16 * (k >> 1) + gid + 8 * (k & 1);
        const float w = ws[k] * down;
        const __half h = __float2half_rn(w);
        const __half l2 = __float2half_rn(w - __half2float(h));
        const int pos = mma_wpos(tl);
        wtab[(2 * tig) * kMmaWRow + pos] = h;
        wtab[(2 * tig + 1) * kMmaWRow + pos] = l2;
    }
    __syncwarp();
    // ---- PV: channel tiles of 16, two k-steps of 16 tokens each ----
    const uint2 bw0 = *reinterpret_cast<const uint2*>(wtab + gid * kMmaWRow + 4 * tig);
    const uint2 bw1 = *reinterpret_cast<const uint2*>(wtab + gid * kMmaWRow + 16 + 4 * tig);
    const uint32_t* vrow = vw_s + tig * DQ;
#pragma unroll
    for (int mh = 0; mh < DQ / 4; ++mh) {
        float d[4][4];  // channel tiles 4mh..4mh+3
#pragma unroll
        for (int kk = 0; kk < 2; ++kk) {
            uint4 vv[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) vv[i] = *reinterpret_cast<const uint4*>(vrow + (16 * kk + 4 * i) * DQ + 4 * mh);
            const uint2 bw = kk == 0 ? bw0 : bw1;
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                const uint32_t w0 = q == 0 ? vv[0].x : q == 1 ? vv[0].y : q == 2 ? vv[0].z : vv[0].w;
                const uint32_t w1 = q == 0 ? vv[1].x : q == 1 ? vv[1].y : q == 2 ? vv[1].z : vv[1].w;
                const uint32_t w2 = q == 0 ? vv[2].x : q == 1 ? vv[2].y : q == 2 ? vv[2].z : vv[2].w;
                const uint32_t w3 = q == 0 ? vv[3].x : q == 1 ? vv[3].y : q == 2 ? vv[3].z : vv[3].w;
                if (kk == 0) mma_codes<true>(d[q], w0, w1, w2, w3, sel, sft, m8, bw.x, bw.y);
                else mma_codes<false>(d[q], w0, w1, w2, w3, sel, sft, m8, bw.x, bw.y);
            }
        }
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            S.acc[4 * mh + q][0] = fmaf(S.acc[4 * mh + q][0], f, d[q][0] + d[q][1]);
            S.acc[4 * mh + q][1] = fmaf(S.acc[4 * mh + q][1], f, d[q][2] + d[q][3]);
        }
    }
    __syncwarp();
}

// Per-warp totals of the tensor-core unit for head tig: m, l and the output
// channels 16mt+gid and 16mt+gid+8 (zero point folded back in).
template <int HD>
__device__ __forceinline__ void mma_finish(MmaState<HD>& S, float& m, float& l, float (&o)[HD / 16][2]) {
    float L = S.l, SW = S.sws, SZ = S.spz;
#pragma unroll
    for (int x = 4; x <= 16; x <<= 1) {
        L += __shfl_xor_sync(0xffffffffu, L, x);
        SW += __shfl_xor_sync(0xffffffffu, SW, x);
        SZ += __shfl_xor_sync(0xffffffffu, SZ, x);
    }
    const float up = pow2f(S.E);
#pragma unroll
    for (int mt = 0; mt < HD / 16; ++mt) {
        o[mt][0] = (S.acc[mt][0] * up - 4.0f * SW) + SZ;
        o[mt][1] = (S.acc[mt][1] * up - 4.0f * SW) + SZ;
    }
    m = S.m;
    l = L;
}

}  // namespace tt
