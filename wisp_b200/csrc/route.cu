// Router: softmax over the expert logits, top-k, optional renormalisation
// (the routing the reference's paged forward takes from vLLM's
// select_experts for Qwen3 / Mixtral, src/wisp/integrations/vllm/
// fused_moe.py:1054-1076), for callers that hand the layer router logits.
//
// One warp per token.  Element e of a row sits in lane e % 32, iteration
// e / 32.  p_e = expf(l_e - max) / sum, where max and sum are reduced over
// the warp: each lane first folds its own elements in iteration order, then
// a fixed xor butterfly (16, 8, 4, 2, 1) combines the lanes -- a fixed order,
// so p does not depend on anything but the row.  Top-k picks the k largest p
// in descending order, ties to the lower expert id; renormalised weights are
// w_j = p_j / (p_0 + ... + p_{k-1}) with the sum and the quotient in double,
// rounded once to fp32 (the correctly rounded renormalisation of the p_j).
#include "common.cuh"

namespace wisp {
namespace {

constexpr int kMaxRouteE = 1024;
constexpr int kPerLane = kMaxRouteE / 32;
constexpr int kWarps = 8;

template <typename TIn>
__device__ __forceinline__ float load_logit(const TIn *p);
template <>
__device__ __forceinline__ float load_logit<float>(const float *p) {
    return *p;
}
template <>
__device__ __forceinline__ float load_logit<__nv_bfloat16>(const __nv_bfloat16 *p) {
    return __bfloat162float(*p);
}

template <typename TIn>
__global__ void __launch_bounds__(kWarps * 32)
    route_topk_kernel(const TIn *logits, int T, int E, int k, int renorm, float *out_w, int32_t *out_ids) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int t = blockIdx.x * kWarps + warp;
    if (t >= T) return;
    const TIn *row = logits + (size_t)t * E;
    const int it = (E + 31) / 32;
    float v[kPerLane];
    float mx = -INFINITY;
#pragma unroll
    for (int i = 0; i < kPerLane; ++i) {
        const int e = i * 32 + lane;
        v[i] = (i < it && e < E) ? load_logit<TIn>(row + e) : -INFINITY;
        mx = fmaxf(mx, v[i]);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    float sum = 0.f;
#pragma unroll
    for (int i = 0; i < kPerLane; ++i) {
        const int e = i * 32 + lane;
        if (i < it && e < E) {
            v[i] = expf(v[i] - mx);
            sum += v[i];
        } else {
            v[i] = -1.f;  // below every probability: never selected
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
#pragma unroll
    for (int i = 0; i < kPerLane; ++i)
        if (v[i] >= 0.f) v[i] = v[i] / sum;
    // top-k: k rounds of a warp arg-max (largest p, then lowest id)
    float sel_p = 0.f;
    int sel_e = 0;
    double tot = 0.0;
    for (int j = 0; j < k; ++j) {
        float bp = -2.f;
        int be = 0x7fffffff;
#pragma unroll
        for (int i = 0; i < kPerLane; ++i) {
            const int e = i * 32 + lane;
            if (v[i] > bp) {  // iterations ascend in e: the first of equal values keeps the lower id
                bp = v[i];
                be = e;
            }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float op = __shfl_xor_sync(0xffffffffu, bp, o);
            const int oe = __shfl_xor_sync(0xffffffffu, be, o);
            if (op > bp || (op == bp && oe < be)) {
                bp = op;
                be = oe;
            }
        }
        // the owner lane retires the element
        if ((be & 31) == lane) {
#pragma unroll
            for (int i = 0; i < kPerLane; ++i)
                if (i * 32 + lane == be) v[i] = -2.f;
        }
        if (lane == j) {
            sel_p = bp;
            sel_e = be;
        }
        tot += (double)bp;  // every lane holds the same running sum, in selection order
    }
    if (lane < k) {
        out_ids[(size_t)t * k + lane] = sel_e;
        out_w[(size_t)t * k + lane] = renorm ? (float)((double)sel_p / tot) : sel_p;
    }
}

}  // namespace
}  // namespace wisp

using namespace wisp;

extern "C" int wisp_route_topk(const void *logits, int32_t logits_bf16, int32_t num_tokens, int32_t num_experts,
                               int32_t top_k, int32_t renormalize, float *topk_weights, int32_t *topk_ids,
                               void *stream) {
    if (num_tokens < 0 || num_experts < 1 || num_experts > kMaxRouteE || top_k < 1 || top_k > 32 ||
        top_k > num_experts)
        return set_error("wisp_route_topk: need 1 <= top_k <= min(32, num_experts), num_experts <= 1024"),
               WISP_ERR_INVALID;
    if (num_tokens == 0) return WISP_OK;
    if (!logits || !topk_weights || !topk_ids) return set_error("wisp_route_topk: NULL tensor"), WISP_ERR_INVALID;
    const dim3 grid((num_tokens + kWarps - 1) / kWarps), block(kWarps * 32);
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    if (logits_bf16)
        route_topk_kernel<__nv_bfloat16><<<grid, block, 0, s>>>(reinterpret_cast<const __nv_bfloat16 *>(logits),
                                                                 num_tokens, num_experts, top_k, renormalize,
                                                                 topk_weights, topk_ids);
    else
        route_topk_kernel<float><<<grid, block, 0, s>>>(reinterpret_cast<const float *>(logits), num_tokens,
                                                        num_experts, top_k, renormalize, topk_weights, topk_ids);
    WISP_CUDA_TRY(cudaGetLastError());
    return WISP_OK;
}
