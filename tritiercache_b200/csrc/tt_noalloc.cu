// tt_noalloc.cu -- fused decode attention for callers that must not allocate.
//
// tt_fused_attention_decode takes its split-KV scratch (per-chunk softmax
// partials and the logits kept for the mean attention weights) from a
// workspace that the library grows with cudaMalloc.  Some callers cannot
// accept that: a process that reserves all device memory up front and treats
// any later CUDA allocation as a failure, a host framework whose allocator
// owns the device memory and forbids cudaMalloc from plug-ins, or a latency-
// critical loop where cudaMalloc/cudaFree (which can synchronise the device)
// is not allowed.  For them this file provides one more entry point whose
// scratch is a fixed array in device memory, declared at file scope.
//
// The array costs kNoAllocScratchBytes of device memory on every GPU where
// the module that holds it is loaded, until the process exits.  CUDA 12 loads
// modules lazily by default, so that happens at the first call of this entry
// point on each device (its cudaGetSymbolAddress is the first use of the
// module): the 32 MiB are reserved then, not when the library is opened.
// Callers that reserve device memory up front make one call at start-up,
// before they reserve and before any stream capture (or run with
// CUDA_MODULE_LOADING=EAGER, which loads it with the library).
#include <climits>
#include <mutex>

#include "tt_attn.cuh"

namespace {

constexpr size_t kNoAllocScratchBytes = (size_t)32 << 20;  // 32 MiB

// Only device code may name this array directly.  In host code its name is a
// host-side stand-in, not a device address, so host code obtains the address
// with cudaGetSymbolAddress (once per device, with that device current).
// That lookup is also what makes a lazily loading runtime load this module
// and reserve the array on the device.  The address is cached per device for
// the life of the process: after a cudaDeviceReset the cached value is stale
// and this entry point must not be called again in that process.
__device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

std::mutex g_mu;
void* g_addr[64] = {};  // device address of g_noalloc_scratch per CUDA device

tt_status scratch_address(int dev, float** out) {
    if (dev < 0 || dev >= 64) return tt::set_error(TT_ERR_UNSUPPORTED, "device ordinal %d out of range", dev);
    std::lock_guard<std::mutex> g(g_mu);
    if (!g_addr[dev]) {
        void* p = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess) return tt::check_cuda(e, "cudaGetSymbolAddress(g_noalloc_scratch)");
        g_addr[dev] = p;
    }
    *out = static_cast<float*>(g_addr[dev]);
    return TT_OK;
}

bool aligned16(const void* p) { return ((uintptr_t)p & 15) == 0; }

}  // namespace

using namespace tt;

extern "C" tt_status tt_fused_attention_decode_noalloc(
    const float* Q, const float* dense_K, const float* dense_V, int dense_count, const int32_t* PBS_K_Packed,
    const void* PBS_K_Scales, const void* PBS_K_Zeroes, const int32_t* PBS_V_Packed, const void* PBS_V_Scales,
    const void* PBS_V_Zeroes, const int64_t* PBS_token_ids, int num_blocks, int num_q_heads, int num_kv_heads,
    int head_dim, float* attn_output, float* mean_attn_weights, int k_group_size, int meta_fp16, void* stream) {
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

    // scratch: [chunks][nq][2] partial (m, l), [chunks][nq][hd] partial outputs,
    // [nq][T] logits -- the same layout the allocating entry point uses
    const int T = dense_count + ntok;
    const int maxch = L.nd + L.np;
    const size_t stride = ((size_t)(T > 0 ? T : 1) + 3) / 4 * 4;  // float4 logit rows
    const size_t ml_floats = ((size_t)maxch * num_q_heads * 2 + 3) / 4 * 4;
    const size_t need = ml_floats + (size_t)maxch * num_q_heads * head_dim + (size_t)num_q_heads * stride + 64;
    if (need * sizeof(float) > kNoAllocScratchBytes)
        return set_error(TT_ERR_INVALID_ARGUMENT,
                         "tt_fused_attention_decode_noalloc: this call needs %zu bytes of scratch but the fixed "
                         "scratch array holds %zu bytes (%d query heads, %d tokens); use "
                         "tt_fused_attention_decode for larger calls",
                         need * sizeof(float), kNoAllocScratchBytes, num_q_heads, T);
    int dev = 0;
    if ((s = check_cuda(cudaGetDevice(&dev), "cudaGetDevice")) != TT_OK) return s;
    float* ws = nullptr;
    if ((s = scratch_address(dev, &ws)) != TT_OK) return s;

    // Nothing in the scratch has to start at zero: the partial kernel writes
    // every (chunk, head) partial and every logit that the finalize kernel reads.
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
