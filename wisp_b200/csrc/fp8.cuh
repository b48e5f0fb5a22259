// Block-quantised FP8 expert compute (W8A8, 128 x 128 weight blocks, the
// format of the reference's FP8 paging path, src/wisp/integrations/vllm/
// fused_moe_fp8.py:61-145): warp-per-row GEMVs on the CUDA cores.
#pragma once
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace wisp {

constexpr int kFp8Block = 128;

struct Fp8Group {
    const uint8_t *xq;         // [T][H] the call's tokens, float8_e4m3fn
    const float *xs;           // [T][H / 128] their group scales
    const uint8_t *w13;        // slot scratch [cap][2I][H] float8_e4m3fn
    const float *s13;          // [cap][2I / 128][H / 128]
    const uint8_t *w2;         // [cap][H][I]
    const float *s2;           // [cap][H / 128][I / 128]
    const int32_t *u_slot;     // this group's unique slots
    const int32_t *u_off;      // n_u + 1 offsets into u_pairs (relative)
    const int32_t *u_pairs;    // absolute pair ids (t*K + k), grouped by unique slot
    const int32_t *nu;         // device count n_u of this group
    const float *topk_w;       // [T*K]
    __nv_bfloat16 *act;        // [T*K][I] SiLU-mul output per pair
    uint8_t *aq;               // [T*K][I] act quantised
    float *as;                 // [T*K][I / 128]
    __nv_bfloat16 *y;          // [T*K][H] weighted expert output per pair
    __nv_bfloat16 *out;        // [T][H]
    int32_t *counters;         // [ceil(H/8)] arrival counters, zero between launches
    int K, H, I, t0, t1;
};

// Per 128-wide group of each row: s = max(amax, 1e-10) / 448 (an IEEE
// division), q = clamp(v / s, +-448) rounded to float8_e4m3fn.
int launch_fp8_quant_rows(const __nv_bfloat16 *v, long rows, int cols, uint8_t *q, float *s,
                          cudaStream_t stream);

// One token group: gate-up + SiLU-mul, quantisation of the activations,
// down x routing weight + routing-order combine (3 kernels).
constexpr int kFp8KernelsPerGroup = 3;
int launch_fp8_group(const Fp8Group &g, int max_nu, cudaStream_t stream);

}  // namespace wisp
