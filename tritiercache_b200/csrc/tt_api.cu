// tt_api.cu -- error plumbing and the stand-alone quantize / dequantize entry
// points of libtritier_b200 (C ABI declared in include/tritier_b200.h).
#include <stdarg.h>
#include <stdio.h>
#include <string.h>

#include <mutex>
#include <vector>

#include "tt_common.cuh"

namespace tt {

static thread_local char g_err[512] = "";

tt_status set_error(tt_status code, const char* fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_err, sizeof(g_err), fmt, ap);
    va_end(ap);
    return code;
}

tt_status check_cuda(cudaError_t err, const char* what) {
    if (err == cudaSuccess) return TT_OK;
    if (err == cudaErrorMemoryAllocation)
        return set_error(TT_ERR_OUT_OF_MEMORY, "%s: %s", what, cudaGetErrorString(err));
    return set_error(TT_ERR_CUDA, "%s: %s", what, cudaGetErrorString(err));
}

tt_status check_launch(const char* what) { return check_cuda(cudaGetLastError(), what); }

// ---------------------------------------------------------------------------
// opt-in launch timing
// ---------------------------------------------------------------------------
struct ProfSlot {
    int kind;
    cudaEvent_t a, b;
};
static std::mutex g_prof_mu;
static bool g_prof_on = false;
static std::vector<ProfSlot> g_prof;
static std::vector<cudaEvent_t> g_prof_pool;

static cudaEvent_t prof_event() {
    cudaEvent_t e = nullptr;
    if (!g_prof_pool.empty()) {
        e = g_prof_pool.back();
        g_prof_pool.pop_back();
    } else {
        cudaEventCreate(&e);
    }
    return e;
}

int prof_begin(int kind, cudaStream_t st) {
    std::lock_guard<std::mutex> g(g_prof_mu);
    if (!g_prof_on) return -1;
    ProfSlot p{kind, prof_event(), prof_event()};
    cudaEventRecord(p.a, st);
    g_prof.push_back(p);
    return (int)g_prof.size() - 1;
}

void prof_end(int slot, cudaStream_t st) {
    if (slot < 0) return;
    std::lock_guard<std::mutex> g(g_prof_mu);
    if (slot < (int)g_prof.size()) cudaEventRecord(g_prof[slot].b, st);
}

// ---------------------------------------------------------------------------
// Kernels
// ---------------------------------------------------------------------------
__global__ void k_quantize_k(const float* __restrict__ K, uint32_t* __restrict__ packed, void* scale,
                             void* zero, int fp16, int H, int D, int grp) {
    quantize_k_block_dev(K, packed, scale, zero, fp16, H, D, grp, blockIdx.x * blockDim.x + threadIdx.x,
                         gridDim.x * blockDim.x);
}

__global__ void k_quantize_v(const float* __restrict__ V, int32_t* __restrict__ packed, void* scale,
                             void* zero, int fp16, int H, int D, int chunk) {
    quantize_v_block_dev(V, packed, scale, zero, fp16, H, D, chunk, blockIdx.x * blockDim.x + threadIdx.x,
                         gridDim.x * blockDim.x);
}

// dequantize_avx2.cpp:24-110 -- one thread per (block, word, head, channel) word,
// writes its 16 tokens: x = fma(code, scale, zero).
__global__ void k_dequantize_k(const int32_t* __restrict__ packed, const void* scale, const void* zero,
                               float* __restrict__ out, int fp16, int nblk, int H, int D, int grp) {
    const int words = grp / 16;
    const size_t n = (size_t)nblk * words * H * D;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        const int c = (int)(i % D);
        const size_t r = i / D;
        const int h = (int)(r % H);
        const size_t bw = r / H;  // block*words + w
        const int w = (int)(bw % words);
        const size_t b = bw / words;
        const size_t midx = (b * H + h) * D + c;
        const float s = load_meta(scale, midx, fp16), z = load_meta(zero, midx, fp16);
        const uint32_t p = (uint32_t)packed[i];
#pragma unroll
        for (int st = 0; st < 16; ++st) {
            const size_t tok = b * grp + w * 16 + st;
            out[(tok * H + h) * D + c] = __fmaf_rn((float)((p >> (2 * st)) & 3u), s, z);
        }
    }
}

// dequantize_avx2.cpp:138-204 -- one thread per (token, head, 16-channel word).
__global__ void k_dequantize_v(const int32_t* __restrict__ packed, const void* scale, const void* zero,
                               float* __restrict__ out, int fp16, int ntok, int H, int D) {
    const int qhd = (D + 15) / 16;
    const size_t n = (size_t)ntok * H * qhd;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        const int g = (int)(i % qhd);
        const size_t th = i / qhd;
        const float s = load_meta(scale, th, fp16), z = load_meta(zero, th, fp16);
        const uint32_t p = (uint32_t)packed[i];
        float* o = out + th * D + g * 16;
#pragma unroll
        for (int k = 0; k < 16; ++k)
            if (g * 16 + k < D) o[k] = __fmaf_rn((float)((p >> (2 * k)) & 3u), s, z);
    }
}

static int grid_for(size_t n, int threads) {
    size_t b = (n + threads - 1) / threads;
    if (b < 1) b = 1;
    if (b > 148 * 16) b = 148 * 16;
    return (int)b;
}

}  // namespace tt

using namespace tt;

extern "C" {

const char* tt_last_error(void) { return g_err; }

tt_status tt_profile_enable(int on) {
    std::lock_guard<std::mutex> g(g_prof_mu);
    g_prof_on = on != 0;
    return TT_OK;
}

tt_status tt_profile_collect(tt_kernel_times* out) {
    if (!out) return set_error(TT_ERR_INVALID_ARGUMENT, "NULL argument.");
    memset(out, 0, sizeof(*out));
    std::lock_guard<std::mutex> g(g_prof_mu);
    tt_status st = TT_OK;
    for (ProfSlot& p : g_prof) {
        float ms = 0.f;
        cudaError_t e = cudaEventSynchronize(p.b);
        if (e == cudaSuccess) e = cudaEventElapsedTime(&ms, p.a, p.b);
        if (e != cudaSuccess && st == TT_OK) st = check_cuda(e, "tt_profile_collect");
        if (p.kind == 0) { out->maintain_ms += ms; out->maintain_launches++; }
        if (p.kind == 1) { out->partial_ms += ms; out->partial_launches++; }
        if (p.kind == 2) { out->finalize_ms += ms; out->finalize_launches++; }
        g_prof_pool.push_back(p.a);
        g_prof_pool.push_back(p.b);
    }
    g_prof.clear();
    return st;
}

const char* tt_version(void) { return "tritier_b200 0.1.0 (sm_100a)"; }

int tt_pointer_is_device(const void* p) {
    if (!p) return 0;
    cudaPointerAttributes a;
    if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
        cudaGetLastError();
        return 0;
    }
    return (a.type == cudaMemoryTypeDevice || a.type == cudaMemoryTypeManaged) ? 1 : 0;
}

tt_status tt_quantize_k_block(const float* K, uint32_t* packed, void* scale, void* zero, int num_heads,
                              int head_dim, int k_group_size, int meta_fp16, void* stream) {
    if (num_heads <= 0 || head_dim <= 0)
        return set_error(TT_ERR_INVALID_ARGUMENT, "num_heads and head_dim must be positive integers.");
    if (k_group_size != 16 && k_group_size != 32)
        return set_error(TT_ERR_INVALID_ARGUMENT, "k_group_size must be 16 or 32.");
    if (!K || !packed || !scale || !zero) return set_error(TT_ERR_INVALID_ARGUMENT, "null pointer argument.");
    const int n = num_heads * head_dim;
    k_quantize_k<<<grid_for(n, 128), 128, 0, (cudaStream_t)stream>>>(K, packed, scale, zero, meta_fp16 ? 1 : 0,
                                                                    num_heads, head_dim, k_group_size);
    return check_launch("quantize_k_block");
}

tt_status tt_quantize_v_block(const float* V, int32_t* packed, void* scale, void* zero, int num_heads,
                              int head_dim, int chunk_size, int meta_fp16, void* stream) {
    if (num_heads <= 0 || head_dim <= 0 || chunk_size <= 0)
        return set_error(TT_ERR_INVALID_ARGUMENT, "num_heads, head_dim and chunk_size must be positive integers.");
    if (head_dim % 16 != 0)
        return set_error(TT_ERR_UNSUPPORTED,
                         "head_dim must be a multiple of 16 (the reference V quantizer reads past the row otherwise).");
    if (!V || !packed || !scale || !zero) return set_error(TT_ERR_INVALID_ARGUMENT, "null pointer argument.");
    const int n = chunk_size * num_heads;
    k_quantize_v<<<grid_for(n, 128), 128, 0, (cudaStream_t)stream>>>(V, packed, scale, zero, meta_fp16 ? 1 : 0,
                                                                    num_heads, head_dim, chunk_size);
    return check_launch("quantize_v_block");
}

tt_status tt_dequantize_k(const int32_t* packed, const void* scale, const void* zero, float* out, int num_blocks,
                          int num_heads, int head_dim, int k_group_size, int meta_fp16, void* stream) {
    if (num_blocks < 0 || num_heads <= 0 || head_dim <= 0)
        return set_error(TT_ERR_INVALID_ARGUMENT, "invalid dequantize_k shape.");
    if (k_group_size != 16 && k_group_size != 32)
        return set_error(TT_ERR_INVALID_ARGUMENT, "k_group_size must be 16 or 32.");
    if (num_blocks == 0) return TT_OK;
    if (!packed || !scale || !zero || !out) return set_error(TT_ERR_INVALID_ARGUMENT, "null pointer argument.");
    const size_t n = (size_t)num_blocks * (k_group_size / 16) * num_heads * head_dim;
    k_dequantize_k<<<grid_for(n, 256), 256, 0, (cudaStream_t)stream>>>(packed, scale, zero, out, meta_fp16 ? 1 : 0,
                                                                      num_blocks, num_heads, head_dim, k_group_size);
    return check_launch("dequantize_k");
}

tt_status tt_dequantize_v(const int32_t* packed, const void* scale, const void* zero, float* out, int total_tokens,
                          int num_heads, int head_dim, int meta_fp16, void* stream) {
    if (total_tokens < 0 || num_heads <= 0 || head_dim <= 0)
        return set_error(TT_ERR_INVALID_ARGUMENT, "invalid dequantize_v shape.");
    if (head_dim % 16 != 0)
        return set_error(TT_ERR_UNSUPPORTED,
                         "head_dim must be a multiple of 16 (the reference V dequantizer writes past the row otherwise).");
    if (total_tokens == 0) return TT_OK;
    if (!packed || !scale || !zero || !out) return set_error(TT_ERR_INVALID_ARGUMENT, "null pointer argument.");
    const size_t n = (size_t)total_tokens * num_heads * ((head_dim + 15) / 16);
    k_dequantize_v<<<grid_for(n, 256), 256, 0, (cudaStream_t)stream>>>(packed, scale, zero, out, meta_fp16 ? 1 : 0,
                                                                      total_tokens, num_heads, head_dim);
    return check_launch("dequantize_v");
}

}  // extern "C"
