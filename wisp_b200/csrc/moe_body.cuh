// Warp-level bodies of the expert compute, shared by the per-group decode
// kernels (decode.cu) and the persistent forward kernel (forward.cu) so both
// run exactly the same arithmetic:
//   h = W13[s] . x[t]   fp32 FMA chain per lane over 16-byte chunks lane, lane+32, ...,
//                       fixed butterfly, stored bf16 (gate rows 0..I-1, up rows I..2I-1)
//   a = silu(g) * u     from the stored values, silu(g) stored bf16 first, a stored bf16
//   y = (W2[s] . a) * w fp32, weight applied in fp32, stored bf16
//   out[t] = sum_k y    k in routing order: bf16 partial sums for top-k <= 4,
//                       fp32 above; stored bf16 (common.cuh: combine_add)
// (vLLM fused_experts' storage points, as called by the reference at
// src/wisp/integrations/vllm/fused_moe.py:1106-1118 and :1155-1167.)
#pragma once
#include "common.cuh"
#include "decode.cuh"

namespace wisp {

// Loads of data that may change while the kernel runs (COHERENT = true: the
// persistent forward kernel, where the copy engine fills slots and other
// CTAs write act) go through L2 only; otherwise weights stream through the
// non-coherent path without L1 allocation.
template <bool COHERENT>
__device__ __forceinline__ uint4 ld_weight16(const void *p) {
    return COHERENT ? ld_cg16(p) : ld_stream16(p);
}
template <bool COHERENT>
__device__ __forceinline__ uint4 ld_act16(const void *p) {
    return COHERENT ? ld_cg16(p) : ld_cached16(p);
}

// act for every pair of unique expert u, row pair (j, I+j); one warp.
// The weight chunks of a batch (up to kGateupBatch per row) are all loaded
// before any arithmetic so that a warp keeps 2 x kGateupBatch x 16 B per lane
// in flight; the FMA order per lane is still chunk 0, 1, 2, ... .
constexpr int kGateupBatch = 8;
template <int MAXP, bool COHERENT = false>
__device__ __forceinline__ void gateup_rowpair(const GroupCompute &a, int u, int j, int lane) {
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
        for (int cb = 0; cb < H; cb += kGateupBatch * 256) {
            uint4 wg[kGateupBatch], wu[kGateupBatch];
#pragma unroll
            for (int m = 0; m < kGateupBatch; ++m) {
                const int c = cb + m * 256 + lane * 8;
                if (c < H) {
                    wg[m] = ld_weight16<COHERENT>(grow + c);
                    wu[m] = ld_weight16<COHERENT>(urow + c);
                }
            }
#pragma unroll
            for (int m = 0; m < kGateupBatch; ++m) {
                const int c = cb + m * 256 + lane * 8;
                if (c < H) {
#pragma unroll
                    for (int i = 0; i < MAXP; ++i) {
                        if (i < np) {
                            const uint4 xv = ld_cached16(xr[i] + c);
                            ag[i] = dot8(wg[m], xv, ag[i]);
                            au[i] = dot8(wu[m], xv, au[i]);
                        }
                    }
                }
            }
        }
#pragma unroll
        for (int i = 0; i < MAXP; ++i) {
            if (i < np) {
                const float g = round_bf16(warp_sum(ag[i]));
                const float v = round_bf16(warp_sum(au[i]));
                if (lane == i) {
                    const float s = silu_stored(g);
                    const int p = a.u_pairs[qb + i];
                    a.act[(size_t)p * I + j] = act_value(s * v);
                }
            }
        }
    }
}

// weighted y for every pair of unique expert u, output row h; one warp.
template <int MAXP, bool COHERENT = false>
__device__ __forceinline__ void down_row(const GroupCompute &a, int u, int h, int lane) {
    const int H = a.H, I = a.I;
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
            const uint4 wv = ld_weight16<COHERENT>(wrow + c);
#pragma unroll
            for (int i = 0; i < MAXP; ++i)
                if (i < np) acc[i] = dot8(wv, ld_act16<COHERENT>(ar[i] + c), acc[i]);
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

// weighted y for every pair of unique expert u, output rows h0..h0+3 (those
// below H); one warp.  Per (row, pair) the same chunk order, FMA chain and
// butterfly as down_row; the four rows' chunks of a batch are loaded before
// any arithmetic (4 x kDownBatch x 16 B per lane in flight).
constexpr int kDownBatch = 4;
template <int MAXQ, bool COHERENT = false>
__device__ __forceinline__ void down_quad(const GroupCompute &a, int u, int h0, int lane) {
    const int H = a.H, I = a.I;
    const int nr = min(4, H - h0);
    const size_t slot = (size_t)a.u_slot[u];
    const __nv_bfloat16 *wbase = a.w2 + slot * (size_t)H * I + (size_t)h0 * I;
    const int q0 = a.u_off[u], q1 = a.u_off[u + 1];
    for (int qb = q0; qb < q1; qb += MAXQ) {
        const int np = min(MAXQ, q1 - qb);
        float acc[4][MAXQ];
        const __nv_bfloat16 *ar[MAXQ];
#pragma unroll
        for (int i = 0; i < MAXQ; ++i) {
            ar[i] = a.act + (size_t)a.u_pairs[qb + (i < np ? i : 0)] * I;
#pragma unroll
            for (int r = 0; r < 4; ++r) acc[r][i] = 0.f;
        }
        for (int cb = 0; cb < I; cb += kDownBatch * 256) {
            uint4 wv[4][kDownBatch];
#pragma unroll
            for (int m = 0; m < kDownBatch; ++m) {
                const int c = cb + m * 256 + lane * 8;
                if (c < I) {
#pragma unroll
                    for (int r = 0; r < 4; ++r)
                        wv[r][m] = ld_weight16<COHERENT>(wbase + (size_t)(r < nr ? r : 0) * I + c);
                }
            }
#pragma unroll
            for (int m = 0; m < kDownBatch; ++m) {
                const int c = cb + m * 256 + lane * 8;
                if (c < I) {
#pragma unroll
                    for (int i = 0; i < MAXQ; ++i) {
                        if (i < np) {
                            const uint4 av = ld_act16<COHERENT>(ar[i] + c);
#pragma unroll
                            for (int r = 0; r < 4; ++r) acc[r][i] = dot8(wv[r][m], av, acc[r][i]);
                        }
                    }
                }
            }
        }
#pragma unroll
        for (int i = 0; i < MAXQ; ++i) {
            if (i < np) {
                const int p = a.u_pairs[qb + i];
                const float wp = a.topk_w[p];
#pragma unroll
                for (int r = 0; r < 4; ++r) {
                    const float s = warp_sum(acc[r][i]);
                    if (lane == 0 && r < nr) a.y[(size_t)p * H + h0 + r] = __float2bfloat16_rn(s * wp);
                }
            }
        }
    }
}

// out[t][hh] = the routing-order sum (combine_add) of the bf16 rows
// y[t K + k][hh], k = 0 .. K-1, rounded to bf16; up to 8 of the loads are in
// flight at once (L2, past L1: the rows come from other blocks).
__device__ __forceinline__ void combine_one(const GroupCompute &a, int t, int hh) {
    const int H = a.H, K = a.K;
    const unsigned short *col = reinterpret_cast<const unsigned short *>(a.y) + (size_t)t * K * H + hh;
    float acc = 0.f;
    for (int k0 = 0; k0 < K; k0 += 8) {
        unsigned short v[8];
#pragma unroll
        for (int j = 0; j < 8; ++j)
            if (k0 + j < K) v[j] = __ldcg(col + (size_t)(k0 + j) * H);
#pragma unroll
        for (int j = 0; j < 8; ++j)
            if (k0 + j < K) acc = combine_add(acc, bf16lo((uint32_t)v[j]), K);
    }
    a.out[(size_t)t * H + hh] = __float2bfloat16_rn(acc);
}

// out rows [h0, h0 + rows) of the group's tokens: sum over k in routing order.
__device__ __forceinline__ void combine_rows(const GroupCompute &a, int h0, int rows, int tid,
                                             int nthreads) {
    const int ntok = a.t1 - a.t0, H = a.H;
    for (int idx = tid; idx < ntok * rows; idx += nthreads) {
        const int hh = h0 + idx % rows;
        if (hh < H) combine_one(a, a.t0 + idx / rows, hh);
    }
}

}  // namespace wisp
