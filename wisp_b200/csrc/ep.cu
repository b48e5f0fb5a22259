// Expert-parallel token dispatch and combine (the exchange itself is NCCL
// all-to-all, issued by the host through torch.distributed).
//
// Rank r owns experts [r * experts_per_rank, (r + 1) * experts_per_rank).
//
//   ep_route_kernel   one warp: for every (token, k) pair p = t * K + k, its
//                     owner rank, a stable counting sort by owner (pairs keep
//                     their order within a rank: the owner's pager sees them
//                     in (source rank, pair) order), the per-rank counts, the
//                     send position of each pair and its (local expert,
//                     weight) record;
//   ep_pack_kernel    one warp per pair: x[t] -> send row pos[p];
//   ep_combine_kernel out[t] = sum over k in routing order of the returned
//                     weighted rows (combine_add: bf16 partial sums for
//                     top-k <= 4, fp32 above), stored bf16 -- the same sum as the
//                     one-GPU forward, so the result is byte-identical to it.
#include <cuda_bf16.h>
#include <stdint.h>

#include "common.cuh"

namespace wisp {
namespace {

constexpr int kRouteMaxRanks = 64;

// counts[world] = number of ids outside [0, world * experts_per_rank).
__global__ void ep_route_kernel(const void *ids, int ids64, const float *w, int P, int e_local, int world,
                                int32_t *meta, long long *counts, int32_t *pos) {
    __shared__ int s_cnt[kRouteMaxRanks], s_off[kRouteMaxRanks];
    const int lane = threadIdx.x;
    for (int d = lane; d < world; d += 32) s_cnt[d] = 0;
    __syncwarp();
    const long long E = (long long)e_local * world;
    int bad = 0;
    for (int p = lane; p < P; p += 32) {
        const long long e = load_id64(ids, ids64, p);
        if (e < 0 || e >= E)
            ++bad;
        else
            atomicAdd(&s_cnt[(int)(e / e_local)], 1);
    }
    __syncwarp();
    bad = __reduce_add_sync(0xffffffffu, bad);
    if (lane == 0) {
        int run = 0;
        for (int d = 0; d < world; ++d) {
            s_off[d] = run;
            run += s_cnt[d];
            counts[d] = s_cnt[d];
        }
        counts[world] = bad;
    }
    __syncwarp();
    if (bad) {  // rejected: no position is valid (the pack kernel skips them)
        for (int p = lane; p < P; p += 32) pos[p] = -1;
        return;
    }
    const unsigned lt = (1u << lane) - 1u;
    for (int p0 = 0; p0 < P; p0 += 32) {
        const int p = p0 + lane;
        int d = -1, loc = 0;
        if (p < P) {
            const long long e = load_id64(ids, ids64, p);
            d = (int)(e / e_local);
            loc = (int)(e - (long long)d * e_local);
        }
        const unsigned same = __match_any_sync(0xffffffffu, d);
        int at = 0;
        if (d >= 0) at = s_off[d] + __popc(same & lt);
        __syncwarp();
        if (d >= 0) {
            pos[p] = at;
            meta[2 * at] = loc;
            meta[2 * at + 1] = __float_as_int(w[p]);
            if ((same & lt) == 0) s_off[d] += __popc(same);  // the group's first lane moves the offset
        }
        __syncwarp();
    }
}

__global__ void ep_pack_kernel(const uint4 *x, const int32_t *pos, int P, int K, int H8, uint4 *send) {
    const int p = blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5);
    if (p >= P) return;
    const int at = pos[p];
    if (at < 0 || at >= P) return;
    const uint4 *src = x + (size_t)(p / K) * H8;
    uint4 *dst = send + (size_t)at * H8;
    for (int c = threadIdx.x & 31; c < H8; c += 32) dst[c] = src[c];
}

__global__ void ep_combine_kernel(const uint4 *y, const int32_t *pos, int T, int K, int H8, uint4 *out) {
    const long i = (long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (long)T * H8) return;
    const int t = (int)(i / H8), c = (int)(i - (long)t * H8);
    float acc[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[j] = 0.f;
    for (int k = 0; k < K; ++k) {
        const uint4 v = y[(size_t)pos[t * K + k] * H8 + c];
        const uint32_t wv[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            acc[2 * j] = combine_add(acc[2 * j], bf16lo(wv[j]), K);
            acc[2 * j + 1] = combine_add(acc[2 * j + 1], bf16hi(wv[j]), K);
        }
    }
    uint32_t o[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const uint32_t lo = __bfloat16_as_ushort(__float2bfloat16_rn(acc[2 * j]));
        const uint32_t hi = __bfloat16_as_ushort(__float2bfloat16_rn(acc[2 * j + 1]));
        o[j] = lo | (hi << 16);
    }
    out[i] = make_uint4(o[0], o[1], o[2], o[3]);
}

}  // namespace
}  // namespace wisp

using namespace wisp;

extern "C" {

int wisp_ep_dispatch(const void *x, const void *topk_ids, int32_t ids_int64, const float *topk_weights,
                     int32_t num_tokens, int32_t top_k, int32_t hidden, int32_t experts_per_rank,
                     int32_t world, void *send_x, int32_t *send_meta, int64_t *send_counts, int32_t *pair_pos,
                     void *stream) {
    if (num_tokens < 0 || top_k < 1 || hidden < 8 || hidden % 8 || experts_per_rank < 1 || world < 1 ||
        world > kRouteMaxRanks)
        return set_error("wisp_ep_dispatch: bad sizes (hidden a multiple of 8, 1 <= world <= 64)"),
               WISP_ERR_INVALID;
    if (!send_counts) return set_error("wisp_ep_dispatch: NULL counts"), WISP_ERR_INVALID;
    const int P = num_tokens * top_k;
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    if (P > 0 && (!x || !topk_ids || !topk_weights || !send_x || !send_meta || !pair_pos))
        return set_error("wisp_ep_dispatch: NULL argument"), WISP_ERR_INVALID;
    ep_route_kernel<<<1, 32, 0, s>>>(topk_ids, ids_int64, topk_weights, P, experts_per_rank, world, send_meta,
                                     reinterpret_cast<long long *>(send_counts), pair_pos);
    WISP_CUDA_TRY(cudaGetLastError());
    if (P > 0) {
        const int warps = 8;
        ep_pack_kernel<<<(P + warps - 1) / warps, warps * 32, 0, s>>>(
            reinterpret_cast<const uint4 *>(x), pair_pos, P, top_k, hidden / 8, reinterpret_cast<uint4 *>(send_x));
        WISP_CUDA_TRY(cudaGetLastError());
    }
    return WISP_OK;
}

int wisp_ep_combine(const void *y_back, const int32_t *pair_pos, int32_t num_tokens, int32_t top_k,
                    int32_t hidden, void *out, void *stream) {
    if (num_tokens < 0 || top_k < 1 || hidden < 8 || hidden % 8)
        return set_error("wisp_ep_combine: bad sizes (hidden a multiple of 8)"), WISP_ERR_INVALID;
    if (num_tokens == 0) return WISP_OK;
    if (!y_back || !pair_pos || !out) return set_error("wisp_ep_combine: NULL argument"), WISP_ERR_INVALID;
    const long n = (long)num_tokens * (hidden / 8);
    ep_combine_kernel<<<(unsigned)((n + 255) / 256), 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
        reinterpret_cast<const uint4 *>(y_back), pair_pos, num_tokens, top_k, hidden / 8,
        reinterpret_cast<uint4 *>(out));
    WISP_CUDA_TRY(cudaGetLastError());
    return WISP_OK;
}

}  // extern "C"
