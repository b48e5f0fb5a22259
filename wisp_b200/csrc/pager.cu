// K1: device-side LRU pager of the paged fused-MoE layer.
//
// One CTA runs one forward's bookkeeping: the first-fit token sub-batching of
// _wisp_forward_cuda_paged (src/wisp/integrations/vllm/fused_moe.py:1102-1140)
// and, for every group in order, the reference's ensure_resident LRU step
// (fused_moe.py:264-358), bit-exact:
//
//   needed  = unique ids of the group, walked in CPython set order
//             (ascending insertion into the interpreter's hash table);
//   missing = needed experts with no slot, in that order;
//   hits   += |needed| - |missing|;  no miss -> clock++, touch, done;
//   free    = empty slots, ascending;
//   victims = occupied slots not needed, ordered by (tick, slot), the first
//             |missing| - |free| of them, appended to free in that order;
//   clock++; each missing expert takes free.pop() (from the END of the list);
//   every needed slot's tick = clock.
//
// Outputs: the state (slot_to_expert, lru_tick, expert_map, clock, counters)
// in place, the slot of every (token, k) pair, per-group unique-slot lists
// with their pairs (CSR) for the compute kernels, and a mailbox in mapped
// pinned host memory with the groups and the page-in list for the host.
#include "pager_body.cuh"

namespace wisp {

size_t pager_smem_bytes(int E, int cap, int T, int K) { return smem_bytes(E, cap, T, K); }

__global__ void __launch_bounds__(kThreads, 1) pager_kernel(const __grid_constant__ PagerParams a) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    pager_body(a, smem_raw);
    pager_finish(a, smem_raw, true);
}

int launch_pager(const PagerParams &p, cudaStream_t stream) {
    const size_t smem = pager_smem_bytes(p.E, p.cap, p.T, p.K);
    // the attribute is per device; remember the largest size set on each
    static int configured_for[64];
    int dev = 0;
    WISP_CUDA_TRY(cudaGetDevice(&dev));
    if (dev < 0 || dev >= 64 || (int)smem > configured_for[dev]) {
        WISP_CUDA_TRY(cudaFuncSetAttribute(pager_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           (int)smem));
        if (dev >= 0 && dev < 64) configured_for[dev] = (int)smem;
    }
    pager_kernel<<<1, kThreads, smem, stream>>>(p);
    WISP_CUDA_TRY(cudaGetLastError());
    return WISP_OK;
}

}  // namespace wisp
