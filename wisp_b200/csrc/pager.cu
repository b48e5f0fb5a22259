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

// ---------------------------------------------------------------------------
// Speculative prefetch (fused_moe.py:360-433), bit-exact:
//   to_load = predicted experts with no slot, in the caller's order; none ->
//             nothing changes (not even the clock);
//   free    = empty slots, ascending;
//   victims = occupied slots whose expert is neither in the layer's last
//             forward's unique set nor predicted, by (tick, slot); when the
//             prediction needs more slots than free + victims it is cut to
//             that many; the first |to_load| - |free| victims are evicted
//             (evictions count) and appended to free;
//   clock++; each expert to load takes free.pop() (from the END), tick =
//   clock.  No miss or hit is counted.
// ---------------------------------------------------------------------------
namespace wisp {
namespace {

constexpr int kPfThreads = 256;

__global__ void __launch_bounds__(kPfThreads, 1) prefetch_kernel(const __grid_constant__ PrefetchParams a) {
    extern __shared__ __align__(16) unsigned char smem[];
    const int tid = threadIdx.x;
    const int E = a.E, cap = a.cap;
    int64_t *tick = reinterpret_cast<int64_t *>(smem);
    int *s2e = reinterpret_cast<int *>(tick + cap);
    int *fre = s2e + cap;           // [cap] free list, then victims
    int *emap = fre + cap;          // [E]
    int *load = emap + E;           // [n]
    __shared__ uint32_t pmask[32], lmask[32];
    __shared__ int s_bad, s_nload, s_nfree, s_need;
    __shared__ long long s_clock;
    if (tid < 32) {
        pmask[tid] = 0;
        lmask[tid] = (tid < (E + 31) / 32) ? a.last_unique[tid] : 0u;
    }
    if (tid == 0) s_bad = 0;
    for (int s = tid; s < cap; s += kPfThreads) {
        tick[s] = a.tick[s];
        s2e[s] = a.s2e[s];
    }
    for (int e = tid; e < E; e += kPfThreads) emap[e] = a.emap[e];
    __syncthreads();
    for (int i = tid; i < a.n; i += kPfThreads) {
        const int e = a.pred[i];
        if (e < 0 || e >= E)
            s_bad = 1;
        else
            atomicOr(&pmask[e >> 5], 1u << (e & 31));
    }
    __syncthreads();
    if (s_bad) {
        if (tid == 0) {
            a.out[1] = 0;
            a.out[0] = WISP_ERR_BAD_EXPERT;
        }
        return;
    }
    if (tid == 0) {
        int nl = 0, nf = 0;
        for (int i = 0; i < a.n; ++i)
            if (emap[a.pred[i]] < 0) load[nl++] = a.pred[i];
        for (int s = 0; s < cap; ++s)
            if (s2e[s] < 0) fre[nf++] = s;
        s_nload = nl;
        s_nfree = nf;
        s_clock = a.hdr[0];
    }
    __syncthreads();
    if (s_nload == 0) {
        if (tid == 0) {
            a.out[1] = 0;
            a.out[0] = WISP_OK;
        }
        return;
    }
    auto eligible = [&](int s) {
        const int e = s2e[s];
        return e >= 0 && !((lmask[e >> 5] >> (e & 31)) & 1u) && !((pmask[e >> 5] >> (e & 31)) & 1u);
    };
    if (tid == 0) {
        int nc = 0;
        for (int s = 0; s < cap; ++s) nc += eligible(s);
        int nl = s_nload;
        if (nl - s_nfree > nc) nl = nc + s_nfree;  // a partial load of the prediction
        s_nload = nl;
        s_need = nl - s_nfree;
    }
    __syncthreads();
    const int nfree = s_nfree, need = s_need, nload = s_nload;
    if (need > 0) {
        for (int s = tid; s < cap; s += kPfThreads) {
            if (!eligible(s)) continue;
            const long long ts = tick[s];
            int rank = 0;
            for (int q = 0; q < cap; ++q) {
                if (!eligible(q)) continue;
                const long long tq = tick[q];
                rank += (tq < ts) || (tq == ts && q < s);
            }
            if (rank < need) fre[nfree + rank] = s;
        }
        __syncthreads();
        if (tid == 0) {
            for (int r = 0; r < need; ++r) {
                const int s = fre[nfree + r];
                emap[s2e[s]] = -1;
                s2e[s] = -1;
            }
        }
        __syncthreads();
    }
    if (tid == 0) {
        const long long clk = s_clock + 1;
        const int total_free = nfree + (need > 0 ? need : 0);
        int *rec = a.out + kMbRec;
        for (int i = 0; i < nload; ++i) {
            const int e = load[i];
            const int s = fre[total_free - 1 - i];  // LIFO pop
            s2e[s] = e;
            emap[e] = s;
            tick[s] = clk;
            const uint32_t gen = a.slot_gen[s] + 1;
            a.slot_gen[s] = gen;
            rec[kMbRec * i + 0] = e;
            rec[kMbRec * i + 1] = s;
            rec[kMbRec * i + 2] = (int)gen;
        }
        s_clock = clk;
    }
    __syncthreads();
    for (int s = tid; s < cap; s += kPfThreads) {
        a.tick[s] = tick[s];
        a.s2e[s] = s2e[s];
    }
    for (int e = tid; e < E; e += kPfThreads) a.emap[e] = emap[e];
    if (tid == 0) {
        a.hdr[0] = s_clock;
        if (need > 0) a.hdr[4] += need;
        a.out[1] = nload;
        __threadfence_system();
        a.out[0] = WISP_OK;
    }
}

}  // namespace

int launch_prefetch(const PrefetchParams &p, cudaStream_t stream) {
    const size_t smem = sizeof(int64_t) * p.cap + sizeof(int) * (2 * (size_t)p.cap + p.E + std::max(p.n, 1));
    static int configured_for[64];
    int dev = 0;
    WISP_CUDA_TRY(cudaGetDevice(&dev));
    if (dev < 0 || dev >= 64 || (int)smem > configured_for[dev]) {
        WISP_CUDA_TRY(cudaFuncSetAttribute(prefetch_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
        if (dev >= 0 && dev < 64) configured_for[dev] = (int)smem;
    }
    prefetch_kernel<<<1, kPfThreads, smem, stream>>>(p);
    WISP_CUDA_TRY(cudaGetLastError());
    return WISP_OK;
}

}  // namespace wisp
