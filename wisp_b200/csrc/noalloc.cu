// Expert compute that allocates nothing: the decode kernels (K3) run on a
// fixed, file-scope device scratch instead of a layer's workspace.
//
// Who needs it: callers that are handed their buffers by a host application
// and may not allocate device memory themselves.  A serving engine that
// reserves nearly all free HBM for its KV cache at start-up leaves a plug-in
// no room for cudaMalloc (and a late cudaMalloc that does succeed shrinks the
// engine's budget behind its back); a latency-critical decode loop cannot
// take cudaMalloc's implicit device synchronisation either.  Such a caller
// passes inputs and outputs and the slot each (token, k) pair reads; this
// entry point keeps its intermediates (per-pair activations, weighted expert
// outputs, the unique-slot lists and the combine's arrival counters) in
// g_static_scratch below.
//
// The array is sized for at most kMaxPairs (token, k) pairs, hidden size
// kMaxHidden and intermediate size kMaxInter (about 6.3 MB).  It is placed in
// a GPU's memory when this file's device code is loaded onto that GPU, and
// CUDA loads device code lazily (the default since CUDA 12.2): on the first
// call on that device, not when the library is loaded.  A call with
// num_tokens == 0 does exactly that set-up (loads the array and the code of
// the kernels a call runs, resolves the array's address) and computes nothing, so a caller that is about to reserve the
// free HBM makes that call first; from then on the GPU holds the array until
// the process exits.  All calls share it and it keeps the last call's
// contents, so calls that overlap on the GPU (on different streams, or from
// different threads without ordering) race.
#include <mutex>

#include "common.cuh"
#include "decode.cuh"

namespace wisp {
namespace {

constexpr int kMaxPairs = 128;     // num_tokens * top_k
constexpr int kMaxHidden = 8192;
constexpr int kMaxInter = 16384;
constexpr int kCsrThreads = 128;   // == kMaxPairs

constexpr size_t align256(size_t v) { return (v + 255) & ~size_t(255); }
constexpr size_t kOffCounters = 0;                                             // int32 [kMaxHidden/8]
constexpr size_t kOffNu = align256(kOffCounters + 4 * (kMaxHidden / 8));       // int32 [1]
constexpr size_t kOffUSlot = align256(kOffNu + 4);                             // int32 [kMaxPairs]
constexpr size_t kOffUOff = align256(kOffUSlot + 4 * kMaxPairs);               // int32 [kMaxPairs+1]
constexpr size_t kOffUPairs = align256(kOffUOff + 4 * (kMaxPairs + 1));        // int32 [kMaxPairs]
constexpr size_t kOffAct = align256(kOffUPairs + 4 * kMaxPairs);               // bf16 [kMaxPairs][kMaxInter]
constexpr size_t kOffY = align256(kOffAct + 2 * (size_t)kMaxPairs * kMaxInter);  // bf16 [kMaxPairs][kMaxHidden]
constexpr size_t kScratchBytes = align256(kOffY + 2 * (size_t)kMaxPairs * kMaxHidden);

static __device__ __align__(256) unsigned char g_static_scratch[kScratchBytes];

// Device address of g_static_scratch per device, resolved once with that
// device current (host code may not use the symbol itself as a pointer).
std::mutex g_addr_mu;
unsigned char *g_addr[64] = {};

// Unique-slot CSR of the pairs (one CTA): pairs whose slot is outside
// [0, num_slots) read no expert and contribute zero (vLLM treats experts the
// expert map does not cover the same way); their weighted outputs are zeroed.
__global__ void __launch_bounds__(kCsrThreads) static_csr_kernel(const int32_t *pair_slots, int P,
                                                                 int num_slots, int H, int T,
                                                                 __nv_bfloat16 *out,
                                                                 unsigned char *base) {
    __shared__ int s_slot[kMaxPairs], s_first[kMaxPairs], s_uidx[kMaxPairs], s_cnt[kMaxPairs],
        s_fill[kMaxPairs];
    __shared__ int s_nu;
    int32_t *nu = reinterpret_cast<int32_t *>(base + kOffNu);
    int32_t *u_slot = reinterpret_cast<int32_t *>(base + kOffUSlot);
    int32_t *u_off = reinterpret_cast<int32_t *>(base + kOffUOff);
    int32_t *u_pairs = reinterpret_cast<int32_t *>(base + kOffUPairs);
    __nv_bfloat16 *y = reinterpret_cast<__nv_bfloat16 *>(base + kOffY);
    const int p = threadIdx.x;
    int s = -1;
    if (p < P) {
        s = pair_slots[p];
        if (s < 0 || s >= num_slots) s = -1;
    }
    s_slot[p] = s;
    s_cnt[p] = 0;
    s_fill[p] = 0;
    __syncthreads();
    // first pair with the same slot
    int first = p;
    if (s >= 0)
        for (int q = 0; q < p; ++q)
            if (s_slot[q] == s) {
                first = q;
                break;
            }
    s_first[p] = first;
    __syncthreads();
    if (p == 0) {
        int n = 0;
        for (int q = 0; q < P; ++q)
            if (s_slot[q] >= 0 && s_first[q] == q) {
                s_uidx[q] = n;
                u_slot[n] = s_slot[q];
                ++n;
            }
        s_nu = n;
        *nu = n;
    }
    __syncthreads();
    int u = -1;
    if (s >= 0) {
        u = s_uidx[first];
        atomicAdd(&s_cnt[u], 1);
    }
    __syncthreads();
    if (p == 0) {
        int run = 0;
        for (int i = 0; i < s_nu; ++i) {
            u_off[i] = run;
            run += s_cnt[i];
        }
        u_off[s_nu] = run;
    }
    __syncthreads();
    if (u >= 0) u_pairs[u_off[u] + atomicAdd(&s_fill[u], 1)] = p;
    // no pair reads an expert: no combine will run, the output is zero
    if (s_nu == 0)
        for (int i = threadIdx.x; i < T * H; i += blockDim.x) out[i] = __float2bfloat16_rn(0.f);
    // zero the weighted outputs of pairs that read no expert
    for (int q = 0; q < P; ++q) {
        if (s_slot[q] >= 0) continue;
        for (int h = threadIdx.x; h < H; h += blockDim.x) y[(size_t)q * H + h] = __float2bfloat16_rn(0.f);
    }
}

int static_scratch_address(int device, unsigned char **out) {
    if (device < 0 || device >= 64) return WISP_ERR_INVALID;
    std::lock_guard<std::mutex> lk(g_addr_mu);
    if (!g_addr[device]) {
        void *ptr = nullptr;
        WISP_CUDA_TRY(cudaGetSymbolAddress(&ptr, g_static_scratch));
        g_addr[device] = reinterpret_cast<unsigned char *>(ptr);
    }
    *out = g_addr[device];
    return WISP_OK;
}

}  // namespace
}  // namespace wisp

using namespace wisp;

extern "C" int wisp_expert_compute_noalloc(int32_t device, const void *x, const void *scratch_w13,
                                           const void *scratch_w2, int32_t num_slots,
                                           const int32_t *pair_slots, const float *topk_weights,
                                           int32_t num_tokens, int32_t top_k, int32_t hidden,
                                           int32_t inter, void *out, void *stream) {
    if (device < 0 || device >= 64)
        return set_error("wisp_expert_compute_noalloc: bad device"), WISP_ERR_INVALID;
    if (num_tokens == 0) {
        // set-up only: place the static array on `device` and resolve its address
        int prev = -1;
        WISP_CUDA_TRY(cudaGetDevice(&prev));
        if (prev != device) WISP_CUDA_TRY(cudaSetDevice(device));
        unsigned char *base = nullptr;
        int rc = static_scratch_address(device, &base);
        // and the code of every kernel a call launches (loading it takes device memory too)
        cudaFuncAttributes fa;
        if (rc == WISP_OK && cudaFuncGetAttributes(&fa, static_csr_kernel) != cudaSuccess) {
            set_error("wisp_expert_compute_noalloc: loading the kernels failed");
            rc = WISP_ERR_CUDA;
        }
        if (rc == WISP_OK) rc = preload_decode_kernels();
        if (prev >= 0 && prev != device) cudaSetDevice(prev);
        return rc;
    }
    if (num_tokens < 0 || top_k < 1 || hidden <= 0 || inter <= 0 || num_slots < 1)
        return set_error("wisp_expert_compute_noalloc: bad sizes"), WISP_ERR_INVALID;
    if ((int64_t)num_tokens * top_k > kMaxPairs || hidden > kMaxHidden || inter > kMaxInter)
        return set_error("wisp_expert_compute_noalloc: sizes exceed the static scratch (at most " +
                         std::to_string(kMaxPairs) + " token x top_k pairs, hidden <= " +
                         std::to_string(kMaxHidden) + ", inter <= " + std::to_string(kMaxInter) + ")"),
               WISP_ERR_INVALID;
    if (hidden % 8 || inter % 8)
        return set_error("wisp_expert_compute_noalloc: hidden and inter must be multiples of 8"),
               WISP_ERR_UNSUPPORTED;
    if (!x || !scratch_w13 || !scratch_w2 || !pair_slots || !topk_weights || !out)
        return set_error("wisp_expert_compute_noalloc: NULL tensor"), WISP_ERR_INVALID;
    for (const void *p : {x, scratch_w13, scratch_w2, (const void *)out})
        if (reinterpret_cast<uintptr_t>(p) & 15u)
            return set_error("wisp_expert_compute_noalloc: x, out and the scratch must be 16-byte aligned"),
                   WISP_ERR_INVALID;
    int prev = -1;
    WISP_CUDA_TRY(cudaGetDevice(&prev));
    if (prev != device) WISP_CUDA_TRY(cudaSetDevice(device));
    unsigned char *base = nullptr;
    int rc = static_scratch_address(device, &base);
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    if (rc == WISP_OK) {
        const int P = num_tokens * top_k;
        // the combine's arrival counters must start at zero
        cudaError_t e = cudaMemsetAsync(base + kOffCounters, 0, sizeof(int32_t) * ((hidden + 7) / 8), s);
        if (e == cudaSuccess) {
            static_csr_kernel<<<1, kCsrThreads, 0, s>>>(pair_slots, P, num_slots, hidden, num_tokens,
                                                        reinterpret_cast<__nv_bfloat16 *>(out), base);
            e = cudaGetLastError();
        }
        if (e != cudaSuccess) {
            set_error(std::string("wisp_expert_compute_noalloc: ") + cudaGetErrorString(e));
            rc = WISP_ERR_CUDA;
        } else {
            GroupCompute gc{};
            gc.x = reinterpret_cast<const __nv_bfloat16 *>(x);
            gc.w13 = reinterpret_cast<const __nv_bfloat16 *>(scratch_w13);
            gc.w2 = reinterpret_cast<const __nv_bfloat16 *>(scratch_w2);
            gc.u_slot = reinterpret_cast<const int32_t *>(base + kOffUSlot);
            gc.u_off = reinterpret_cast<const int32_t *>(base + kOffUOff);
            gc.u_pairs = reinterpret_cast<const int32_t *>(base + kOffUPairs);
            gc.nu = reinterpret_cast<const int32_t *>(base + kOffNu);
            gc.topk_w = topk_weights;
            gc.act = reinterpret_cast<__nv_bfloat16 *>(base + kOffAct);
            gc.y = reinterpret_cast<__nv_bfloat16 *>(base + kOffY);
            gc.out = reinterpret_cast<__nv_bfloat16 *>(out);
            gc.counters = reinterpret_cast<int32_t *>(base + kOffCounters);
            gc.K = top_k;
            gc.H = hidden;
            gc.I = inter;
            gc.t0 = 0;
            gc.t1 = num_tokens;
            rc = launch_decode_group(gc, P < num_slots ? P : num_slots, s);
        }
    }
    if (prev >= 0 && prev != device) cudaSetDevice(prev);
    return rc;
}
