// Block-quantised FP8 expert compute on the CUDA cores (see fp8.cuh).
//
// The arithmetic of vLLM's block-FP8 fused_experts, which the reference's FP8
// paging path calls (src/wisp/integrations/vllm/fused_moe_fp8.py:302-312):
//   xq, xs = quant(x)                       per 128-wide group of a row
//   h[n]   = sum_b (xq_b . W13q[n]_b) * xs_b * S13[n / 128][b]   (fp32, stored bf16)
//   a      = bf16(silu(g)) * u              (stored bf16)
//   aq, as = quant(a)
//   y[n]   = (sum_b (aq_b . W2q[n]_b) * as_b * S2[n / 128][b]) * w   (fp32, stored bf16)
//   out[t] = routing-order sum over k (combine_add)
// Each lane owns 16-byte chunks lane*16 + 512*m of a row (every chunk inside
// one 128-group), multiplies the fp8 pairs exactly in fp32 (4-bit
// significands), scales each chunk's dot product by its group's two scales
// and adds it to its fp32 sum; the warp reduces with the fixed butterfly.
#include <cuda_fp16.h>
#include <cuda_fp8.h>

#include "common.cuh"
#include "fp8.cuh"

namespace wisp {
namespace {

constexpr int kWarps = 8;
constexpr float kFp8Max = 448.0f;

__device__ __forceinline__ float2 fp8x2_to_float2(uint32_t two) {
    const __half2_raw r = __nv_cvt_fp8x2_to_halfraw2((__nv_fp8x2_storage_t)(two & 0xffffu), __NV_E4M3);
    return __half22float2(*reinterpret_cast<const __half2 *>(&r));
}

// 16 fp8 products summed in element order (exact products, fp32 sums).
__device__ __forceinline__ float dot16_fp8(const uint4 &w, const uint4 &x) {
    const uint32_t wv[4] = {w.x, w.y, w.z, w.w}, xv[4] = {x.x, x.y, x.z, x.w};
    float acc = 0.f;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
#pragma unroll
        for (int hlf = 0; hlf < 2; ++hlf) {
            const float2 a = fp8x2_to_float2(wv[j] >> (16 * hlf));
            const float2 b = fp8x2_to_float2(xv[j] >> (16 * hlf));
            acc = fmaf(a.x, b.x, acc);
            acc = fmaf(a.y, b.y, acc);
        }
    }
    return acc;
}

// One warp per 128-wide group of a row.
__global__ void __launch_bounds__(kWarps * 32)
    fp8_quant_kernel(const __nv_bfloat16 *v, long groups, int gpr, uint8_t *q, float *s) {
    const long gid = (long)blockIdx.x * kWarps + (threadIdx.x >> 5);
    if (gid >= groups) return;
    const int lane = threadIdx.x & 31;
    const __nv_bfloat16 *src = v + gid * kFp8Block + lane * 4;  // groups are consecutive in the row-major array
    const uint2 raw = *reinterpret_cast<const uint2 *>(src);
    float f[4] = {bf16lo(raw.x), bf16hi(raw.x), bf16lo(raw.y), bf16hi(raw.y)};
    float amax = fmaxf(fmaxf(fabsf(f[0]), fabsf(f[1])), fmaxf(fabsf(f[2]), fabsf(f[3])));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    const float sc = fmaxf(amax, 1e-10f) / kFp8Max;  // a division, as vLLM's quantiser computes it
    uint32_t packed = 0;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const float c = fminf(fmaxf(f[i] / sc, -kFp8Max), kFp8Max);
        packed |= (uint32_t)__nv_cvt_float_to_fp8(c, __NV_SATFINITE, __NV_E4M3) << (8 * i);
    }
    *reinterpret_cast<uint32_t *>(q + gid * kFp8Block + lane * 4) = packed;
    if (lane == 0) s[gid] = sc;
    (void)gpr;
}

template <int MAXP>
__global__ void __launch_bounds__(kWarps * 32) fp8_gateup_kernel(Fp8Group a) {
    const int u = blockIdx.y;
    if (u >= *a.nu) return;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int j = blockIdx.x * kWarps + warp;
    if (j >= a.I) return;
    const int H = a.H, I = a.I, K = a.K, HB = H / kFp8Block;
    const size_t slot = (size_t)a.u_slot[u];
    const uint8_t *grow = a.w13 + slot * (size_t)(2 * I) * H + (size_t)j * H;
    const uint8_t *urow = grow + (size_t)I * H;
    const float *sg = a.s13 + slot * (size_t)(2 * I / kFp8Block) * HB + (size_t)(j / kFp8Block) * HB;
    const float *su = a.s13 + slot * (size_t)(2 * I / kFp8Block) * HB + (size_t)((I + j) / kFp8Block) * HB;
    const int q0 = a.u_off[u], q1 = a.u_off[u + 1];
    for (int qb = q0; qb < q1; qb += MAXP) {
        const int np = min(MAXP, q1 - qb);
        float ag[MAXP], au[MAXP];
        const uint8_t *xr[MAXP];
        const float *xsr[MAXP];
#pragma unroll
        for (int i = 0; i < MAXP; ++i) {
            ag[i] = 0.f;
            au[i] = 0.f;
            const int t = a.u_pairs[qb + (i < np ? i : 0)] / K;
            xr[i] = a.xq + (size_t)t * H;
            xsr[i] = a.xs + (size_t)t * HB;
        }
#pragma unroll 2
        for (int c = lane * 16; c < H; c += 512) {
            const int kb = c / kFp8Block;
            const uint4 wg = ld_stream16(grow + c), wu = ld_stream16(urow + c);
            const float gs = sg[kb], us = su[kb];
#pragma unroll
            for (int i = 0; i < MAXP; ++i) {
                if (i < np) {
                    const uint4 xv = ld_cached16(xr[i] + c);
                    const float xsv = xsr[i][kb];
                    ag[i] += dot16_fp8(wg, xv) * xsv * gs;
                    au[i] += dot16_fp8(wu, xv) * xsv * us;
                }
            }
        }
#pragma unroll
        for (int i = 0; i < MAXP; ++i) {
            if (i < np) {
                const float g = round_bf16(warp_sum(ag[i]));
                const float v = round_bf16(warp_sum(au[i]));
                if (lane == i) {
                    const int p = a.u_pairs[qb + i];
                    a.act[(size_t)p * I + j] = __float2bfloat16_rn(silu_stored(g) * v);
                }
            }
        }
    }
}

template <int MAXP>
__global__ void __launch_bounds__(kWarps * 32) fp8_down_combine_kernel(Fp8Group a) {
    __shared__ int s_last;
    const int u = blockIdx.y;
    const int nu = *a.nu;
    if (u >= nu) return;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int h = blockIdx.x * kWarps + warp;
    const int H = a.H, I = a.I, IB = I / kFp8Block;
    if (h < H) {
        const size_t slot = (size_t)a.u_slot[u];
        const uint8_t *wrow = a.w2 + slot * (size_t)H * I + (size_t)h * I;
        const float *srow = a.s2 + slot * (size_t)(H / kFp8Block) * IB + (size_t)(h / kFp8Block) * IB;
        const int q0 = a.u_off[u], q1 = a.u_off[u + 1];
        for (int qb = q0; qb < q1; qb += MAXP) {
            const int np = min(MAXP, q1 - qb);
            float acc[MAXP];
#pragma unroll
            for (int i = 0; i < MAXP; ++i) acc[i] = 0.f;
            for (int c = lane * 16; c < I; c += 512) {
                const int kb = c / kFp8Block;
                const uint4 wv = ld_stream16(wrow + c);
                const float ws = srow[kb];
#pragma unroll
                for (int i = 0; i < MAXP; ++i) {
                    if (i < np) {
                        const int p = a.u_pairs[qb + i];
                        const uint4 av = ld_cached16(a.aq + (size_t)p * I + c);
                        acc[i] += dot16_fp8(wv, av) * a.as[(size_t)p * IB + kb] * ws;
                    }
                }
            }
#pragma unroll
            for (int i = 0; i < MAXP; ++i) {
                if (i < np) {
                    const float sum = warp_sum(acc[i]);
                    if (lane == i) {
                        const int p = a.u_pairs[qb + i];
                        a.y[(size_t)p * H + h] = __float2bfloat16_rn(sum * a.topk_w[p]);
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
    const int h0 = blockIdx.x * kWarps, ntok = a.t1 - a.t0, K = a.K;
    for (int idx = threadIdx.x; idx < ntok * kWarps; idx += blockDim.x) {
        const int t = a.t0 + idx / kWarps, hh = h0 + idx % kWarps;
        if (hh >= H) continue;
        float s = 0.f;
        for (int k = 0; k < K; ++k) s = combine_add(s, __bfloat162float(__ldcg(a.y + ((size_t)t * K + k) * H + hh)), K);
        a.out[(size_t)t * H + hh] = __float2bfloat16_rn(s);
    }
    if (threadIdx.x == 0) a.counters[blockIdx.x] = 0;
}

template <int MAXP>
int launch_variant(const Fp8Group &g, int max_nu, cudaStream_t stream) {
    const dim3 block(kWarps * 32);
    fp8_gateup_kernel<MAXP><<<dim3((g.I + kWarps - 1) / kWarps, max_nu), block, 0, stream>>>(g);
    WISP_CUDA_TRY(cudaGetLastError());
    const long p0 = (long)g.t0 * g.K, rows = (long)(g.t1 - g.t0) * g.K;
    int rc = launch_fp8_quant_rows(g.act + p0 * g.I, rows, g.I, g.aq + p0 * g.I, g.as + p0 * (g.I / kFp8Block),
                                   stream);
    if (rc) return rc;
    fp8_down_combine_kernel<MAXP><<<dim3((g.H + kWarps - 1) / kWarps, max_nu), block, 0, stream>>>(g);
    WISP_CUDA_TRY(cudaGetLastError());
    return WISP_OK;
}

}  // namespace

int launch_fp8_quant_rows(const __nv_bfloat16 *v, long rows, int cols, uint8_t *q, float *s, cudaStream_t stream) {
    const long groups = rows * (cols / kFp8Block);
    if (groups <= 0) return WISP_OK;
    fp8_quant_kernel<<<(unsigned)((groups + kWarps - 1) / kWarps), kWarps * 32, 0, stream>>>(v, groups,
                                                                                           cols / kFp8Block, q, s);
    WISP_CUDA_TRY(cudaGetLastError());
    return WISP_OK;
}

int launch_fp8_group(const Fp8Group &g, int max_nu, cudaStream_t stream) {
    if (max_nu <= 0 || g.t1 <= g.t0) return WISP_OK;
    const int ntok = g.t1 - g.t0;
    if (ntok <= 1) return launch_variant<1>(g, max_nu, stream);
    if (ntok <= 2) return launch_variant<2>(g, max_nu, stream);
    if (ntok <= 4) return launch_variant<4>(g, max_nu, stream);
    return launch_variant<8>(g, max_nu, stream);
}

}  // namespace wisp
