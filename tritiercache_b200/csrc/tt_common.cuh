// tt_common.cuh -- shared device/host helpers of libtritier_b200.
//
// Numerics that must be bit-exact with the reference's AVX2 kernels live
// here: the min/max operand rules of MINPS/MAXPS versus std::min/std::max,
// IEEE division, round-to-nearest-even float->int with CVTPS2DQ's
// out-of-range value, and binary16 metadata rounding (RNE, as F16C's
// _mm256_cvtps_ph(v, 0)).  The library is compiled without --use_fast_math,
// so '/' and the conversions below are correctly rounded.
#pragma once
#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <stdint.h>
#include <math.h>

#include "../../include/tritier_b200.h"

#define TT_WARP 32

namespace tt {

// ---------------------------------------------------------------------------
// Host-side error plumbing (definitions in tt_api.cu)
// ---------------------------------------------------------------------------
tt_status set_error(tt_status code, const char* fmt, ...);
tt_status check_cuda(cudaError_t err, const char* what);
tt_status check_launch(const char* what);

// Opt-in launch timing (tt_profile_enable): kind 0 maintain, 1 partial, 2 finalize.
int prof_begin(int kind, cudaStream_t st);   // returns a slot or -1 when disabled
void prof_end(int slot, cudaStream_t st);

// ---------------------------------------------------------------------------
// Lane semantics of the reference's vector code
// ---------------------------------------------------------------------------
__device__ __forceinline__ float vmin_ps(float a, float b) { return a < b ? a : b; }  // MINPS
__device__ __forceinline__ float vmax_ps(float a, float b) { return a > b ? a : b; }  // MAXPS
__device__ __forceinline__ float std_min(float a, float b) { return b < a ? b : a; }  // std::min
__device__ __forceinline__ float std_max(float a, float b) { return a < b ? b : a; }  // std::max

// CVTPS2DQ with the default rounding mode: RNE, INT_MIN when out of range or NaN.
__device__ __forceinline__ int cvtps_epi32(float x) {
    if (!(x >= -2147483648.0f && x < 2147483648.0f)) return (int)0x80000000;
    return __float2int_rn(x);
}

// 2-bit code of a value, exactly as quantize_{k,v}_avx2: clamp(rne((x-mn)/scale), 0, 3).
__device__ __forceinline__ uint32_t quant_code(float x, float mn, float scale) {
    int q = cvtps_epi32(__fdiv_rn(__fsub_rn(x, mn), scale));
    q = q < 0 ? 0 : q;
    q = q > 3 ? 3 : q;
    return (uint32_t)q;
}

// Metadata storage: float or IEEE binary16 bits.
__device__ __forceinline__ void store_meta(void* base, size_t idx, float v, int fp16) {
    if (fp16) reinterpret_cast<uint16_t*>(base)[idx] = __half_as_ushort(__float2half_rn(v));
    else reinterpret_cast<float*>(base)[idx] = v;
}
__device__ __forceinline__ float load_meta(const void* base, size_t idx, int fp16) {
    if (fp16) return __half2float(__ushort_as_half(reinterpret_cast<const uint16_t*>(base)[idx]));
    return reinterpret_cast<const float*>(base)[idx];
}

// ---------------------------------------------------------------------------
// Block-cooperative quantizers (one K block / one V chunk), bit-exact with
// csrc/cpu/quantize_k_avx2.cpp:26-110 and csrc/cpu/quantize_v_avx2.cpp:44-108.
// K:   src row stride = H*D floats; thread per (head, channel).
// V:   thread per (token, head); head_dim % 16 == 0.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void quantize_k_block_dev(const float* __restrict__ K, uint32_t* __restrict__ packed,
                                                     void* scale_out, void* zero_out, int fp16, int H, int D,
                                                     int grp, int tid, int nthreads) {
    const int row = H * D;
    const int c_vec_end = (D / 8) * 8;
    const int words = grp / 16;
    for (int hc = tid; hc < H * D; hc += nthreads) {
        const int h = hc / D, c = hc - h * D;
        const float* src = K + (size_t)h * D + c;
        const bool vec = c < c_vec_end;
        float mn = INFINITY, mx = -INFINITY;
        for (int t = 0; t < grp; ++t) {
            float x = src[(size_t)t * row];
            if (vec) { mn = vmin_ps(mn, x); mx = vmax_ps(mx, x); }
            else { mn = std_min(mn, x); mx = std_max(mx, x); }
        }
        float d3 = __fdiv_rn(__fsub_rn(mx, mn), 3.0f);
        float scale = vec ? vmax_ps(d3, 1e-9f) : std_max(d3, 1e-9f);
        store_meta(scale_out, hc, scale, fp16);
        store_meta(zero_out, hc, mn, fp16);
        for (int w = 0; w < words; ++w) {
            uint32_t bits = 0;
#pragma unroll
            for (int st = 0; st < 16; ++st)
                bits |= quant_code(src[(size_t)(w * 16 + st) * row], mn, scale) << (2 * st);
            packed[((size_t)w * H + h) * D + c] = bits;
        }
    }
}

__device__ __forceinline__ void quantize_v_block_dev(const float* __restrict__ V, int32_t* __restrict__ packed,
                                                     void* scale_out, void* zero_out, int fp16, int H, int D,
                                                     int chunk, int tid, int nthreads) {
    const int qhd = D / 16;
    for (int th = tid; th < chunk * H; th += nthreads) {
        const float* v = V + (size_t)th * D;  // (t*H + h)*D
        float mn = INFINITY, mx = -INFINITY;
        for (int c = 0; c < D; c += 8) {
            // hmin8 / hmax8 tree (quantize_v_avx2.cpp:7-23)
            float m0 = vmin_ps(v[c + 0], v[c + 4]), m1 = vmin_ps(v[c + 1], v[c + 5]);
            float m2 = vmin_ps(v[c + 2], v[c + 6]), m3 = vmin_ps(v[c + 3], v[c + 7]);
            float a0 = vmin_ps(m0, m2), a1 = vmin_ps(m1, m3);
            mn = std_min(mn, vmin_ps(a0, a1));
            float x0 = vmax_ps(v[c + 0], v[c + 4]), x1 = vmax_ps(v[c + 1], v[c + 5]);
            float x2 = vmax_ps(v[c + 2], v[c + 6]), x3 = vmax_ps(v[c + 3], v[c + 7]);
            float b0 = vmax_ps(x0, x2), b1 = vmax_ps(x1, x3);
            mx = std_max(mx, vmax_ps(b0, b1));
        }
        float scale = std_max(__fdiv_rn(__fsub_rn(mx, mn), 3.0f), 1e-9f);
        store_meta(scale_out, th, scale, fp16);
        store_meta(zero_out, th, mn, fp16);
        for (int g = 0; g < qhd; ++g) {
            uint32_t word = 0;
#pragma unroll
            for (int i = 0; i < 16; ++i) word |= quant_code(v[g * 16 + i], mn, scale) << (2 * i);
            packed[(size_t)th * qhd + g] = (int32_t)word;
        }
    }
}

// ---------------------------------------------------------------------------
// Misc
// ---------------------------------------------------------------------------
__host__ __device__ __forceinline__ int ceil_div(int a, int b) { return (a + b - 1) / b; }

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// Streaming loads of read-once cache data: do not keep them in L1.
__device__ __forceinline__ int4 ldg_stream_i4(const void* p) {
    int4 r;
    asm volatile("ld.global.nc.L1::no_allocate.v4.s32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "l"(p));
    return r;
}
__device__ __forceinline__ float4 ldg_stream_f4(const void* p) {
    float4 r;
    asm volatile("ld.global.nc.L1::no_allocate.v4.f32 {%0,%1,%2,%3}, [%4];"
                 : "=f"(r.x), "=f"(r.y), "=f"(r.z), "=f"(r.w) : "l"(p));
    return r;
}

}  // namespace tt
