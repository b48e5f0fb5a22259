// Slot-indexed expert compute, warp-per-row GEMV variant (decode, and the
// fallback for small token groups).
#pragma once
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace wisp {

struct GroupCompute {
    const __nv_bfloat16 *x;    // [T][H] token rows
    const __nv_bfloat16 *w13;  // slot scratch [cap][2I][H]
    const __nv_bfloat16 *w2;   // slot scratch [cap][H][I]
    const int32_t *u_slot;     // this group's unique slots (n_u)
    const int32_t *u_off;      // n_u + 1 offsets into u_pairs (relative)
    const int32_t *u_pairs;    // absolute pair ids (t*K + k), grouped by unique slot
    const int32_t *nu;         // device count n_u of this group
    const float *topk_w;       // [T*K]
    __nv_bfloat16 *act;        // [T*K][I] SiLU-mul output per pair
    __nv_bfloat16 *y;          // [T*K][H] weighted expert output per pair
    __nv_bfloat16 *out;        // [T][H]
    int32_t *counters;         // [ceil(H/8)] arrival counters, zero between launches
    int K, H, I, t0, t1;
};

// Launch the two decode kernels for one token group; grid y = max_nu CTAs per
// row block (CTAs beyond the device count n_u exit at once).
// Launches kDecodeKernelsPerGroup kernels: gate-up + SiLU-mul, then down + combine.
constexpr int kDecodeKernelsPerGroup = 2;
int launch_decode_group(const GroupCompute &g, int max_nu, cudaStream_t stream);

// Load the decode kernels' code onto the current device now (CUDA loads
// device code lazily, at a kernel's first launch, and loading takes device
// memory); for callers that must not take device memory later.
int preload_decode_kernels();

}  // namespace wisp
