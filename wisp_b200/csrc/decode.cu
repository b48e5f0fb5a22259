// K3: decode-path expert compute from the slot scratch (memory-bound GEMV).
//
// Semantics are vLLM fused_experts' as the reference calls it with
// expert_map (src/wisp/integrations/vllm/fused_moe.py:1106-1118, 1155-1167),
// per (token t, routed position k) with slot s and weight w:
//   h = W13[s] . x[t]           fp32 accumulate, stored bf16 (gate rows 0..I-1, up rows I..2I-1)
//   a = silu(g) * u             fp32 from the stored values, stored bf16
//   y = (W2[s] . a) * w         fp32 accumulate, weight applied in fp32, stored bf16
//   out[t] = sum_k y (k in routing order), fp32, stored bf16
//
// Every dot product is computed by one warp: lane L covers the 16-byte
// chunks L, L+32, L+64, ... of the row, FMA-chained in element order, then a
// fixed butterfly reduction.  The arithmetic of a (t, k) pair therefore does
// not depend on which other pairs share its group, its slot, or the cap.
//
// gateup_silu_kernel: grid (ceil(I/8), max_nu); warp w of block (bx, u)
//   handles row pair (j, I+j), j = 8*bx + w, of unique expert u, for all of
//   u's pairs.  Reads each weight row once (streamed, evict-first).
// down_combine_kernel: grid (ceil(H/8), max_nu); warp w handles row h of
//   W2[u] for all of u's pairs and stores the weighted result y.  The last
//   CTA to finish a row block (arrival counter) sums the group's tokens over
//   k in routing order for those 8 rows and writes out.
#include "common.cuh"
#include "decode.cuh"

namespace wisp {

namespace {

constexpr int kWarps = 8;
constexpr int kRowsPerBlock = kWarps;

template <int MAXP>
__global__ void __launch_bounds__(kWarps * 32) gateup_silu_kernel(GroupCompute a) {
    const int u = blockIdx.y;
    if (u >= *a.nu) return;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int j = blockIdx.x * kRowsPerBlock + warp;
    if (j >= a.I) return;
    const int H = a.H, I = a.I, K = a.K;
    const size_t slot = (size_t)a.u_slot[u];
    const __nv_bfloat16 *grow = a.w13 + slot * (size_t)(2 * I) * H + (size_t)j * H;
    const __nv_bfloat16 *urow = grow + (size_t)I * H;
    const int q0 = a.u_off[u], q1 = a.u_off[u + 1];
    for (int qb = q0; qb < q1; qb += MAXP) {
        const int np = min(MAXP, q1 - qb);
        float ag[MAXP], au[MAXP];
        const __nv_bfloat16 *xr[MAXP];
#pragma unroll
        for (int i = 0; i < MAXP; ++i) {
            ag[i] = 0.f;
            au[i] = 0.f;
            int p = a.u_pairs[qb + (i < np ? i : 0)];
            xr[i] = a.x + (size_t)(p / K) * H;
        }
#pragma unroll 4
        for (int c = lane * 8; c < H; c += 256) {
            const uint4 wg = ld_stream16(grow + c);
            const uint4 wu = ld_stream16(urow + c);
#pragma unroll
            for (int i = 0; i < MAXP; ++i) {
                if (i < np) {
                    const uint4 xv = ld_cached16(xr[i] + c);
                    ag[i] = dot8(wg, xv, ag[i]);
                    au[i] = dot8(wu, xv, au[i]);
                }
            }
        }
#pragma unroll
        for (int i = 0; i < MAXP; ++i) {
            if (i < np) {
                const float g = round_bf16(warp_sum(ag[i]));
                const float v = round_bf16(warp_sum(au[i]));
                if (lane == i) {
                    const float s = g / (1.0f + expf(-g));
                    const int p = a.u_pairs[qb + i];
                    a.act[(size_t)p * I + j] = __float2bfloat16_rn(s * v);
                }
            }
        }
    }
}

template <int MAXP>
__global__ void __launch_bounds__(kWarps * 32) down_combine_kernel(GroupCompute a) {
    __shared__ int s_last;
    const int u = blockIdx.y;
    const int nu = *a.nu;
    if (u >= nu) return;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int H = a.H, I = a.I, K = a.K;
    const int h = blockIdx.x * kRowsPerBlock + warp;
    if (h < H) {
        const size_t slot = (size_t)a.u_slot[u];
        const __nv_bfloat16 *wrow = a.w2 + slot * (size_t)H * I + (size_t)h * I;
        const int q0 = a.u_off[u], q1 = a.u_off[u + 1];
        for (int qb = q0; qb < q1; qb += MAXP) {
            const int np = min(MAXP, q1 - qb);
            float acc[MAXP];
            const __nv_bfloat16 *ar[MAXP];
#pragma unroll
            for (int i = 0; i < MAXP; ++i) {
                acc[i] = 0.f;
                ar[i] = a.act + (size_t)a.u_pairs[qb + (i < np ? i : 0)] * I;
            }
#pragma unroll 4
            for (int c = lane * 8; c < I; c += 256) {
                const uint4 wv = ld_stream16(wrow + c);
#pragma unroll
                for (int i = 0; i < MAXP; ++i)
                    if (i < np) acc[i] = dot8(wv, ld_cached16(ar[i] + c), acc[i]);
            }
#pragma unroll
            for (int i = 0; i < MAXP; ++i) {
                if (i < np) {
                    const float s = warp_sum(acc[i]);
                    if (lane == i) {
                        const int p = a.u_pairs[qb + i];
                        a.y[(size_t)p * H + h] = __float2bfloat16_rn(s * a.topk_w[p]);
                    }
                }
            }
        }
    }
    // arrival: the last of the nu CTAs of this row block does the combine
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) s_last = (atomicAdd(&a.counters[blockIdx.x], 1) == nu - 1);
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    const int h0 = blockIdx.x * kRowsPerBlock;
    const int ntok = a.t1 - a.t0;
    for (int idx = threadIdx.x; idx < ntok * kRowsPerBlock; idx += blockDim.x) {
        const int t = a.t0 + idx / kRowsPerBlock;
        const int hh = h0 + idx % kRowsPerBlock;
        if (hh >= H) continue;
        float acc = 0.f;
        for (int k = 0; k < K; ++k)
            acc += __bfloat162float(__ldcg(a.y + ((size_t)t * K + k) * H + hh));
        a.out[(size_t)t * H + hh] = __float2bfloat16_rn(acc);
    }
    if (threadIdx.x == 0) a.counters[blockIdx.x] = 0;
}

template <int MAXP>
int launch_variant(const GroupCompute &g, int max_nu, cudaStream_t stream) {
    dim3 block(kWarps * 32);
    dim3 g1((g.I + kRowsPerBlock - 1) / kRowsPerBlock, max_nu);
    gateup_silu_kernel<MAXP><<<g1, block, 0, stream>>>(g);
    WISP_CUDA_TRY(cudaGetLastError());
    dim3 g2((g.H + kRowsPerBlock - 1) / kRowsPerBlock, max_nu);
    down_combine_kernel<MAXP><<<g2, block, 0, stream>>>(g);
    WISP_CUDA_TRY(cudaGetLastError());
    return WISP_OK;
}

}  // namespace

int launch_decode_group(const GroupCompute &g, int max_nu, cudaStream_t stream) {
    if (max_nu <= 0 || g.t1 <= g.t0) return WISP_OK;
    const int ntok = g.t1 - g.t0;
    if (ntok <= 1) return launch_variant<1>(g, max_nu, stream);
    if (ntok <= 2) return launch_variant<2>(g, max_nu, stream);
    if (ntok <= 4) return launch_variant<4>(g, max_nu, stream);
    if (ntok <= 8) return launch_variant<8>(g, max_nu, stream);
    return launch_variant<16>(g, max_nu, stream);
}

}  // namespace wisp
