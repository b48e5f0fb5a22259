// Device pager (K1) interface shared by the runtime.
#pragma once
#include <stddef.h>
#include <stdint.h>

#include <cuda_runtime.h>

namespace wisp {

// Mailbox (mapped pinned host memory, int32 words) written by the pager:
//   [0] status  [1] groups G  [2] misses  [3] failing group  [4] sum of unique experts
//   [kMbHeader ...]            group first tokens, G+1 entries (last = T)
//   [kMbHeader + T + 1 ...]    unique experts per group, G entries
//   [mailbox_miss_offset(T)..] page-in records {expert, slot, group, wait_group}
constexpr int kMbHeader = 8;
inline __host__ __device__ long mailbox_miss_offset(int T) {
    return ((kMbHeader + 2L * T + 1 + 3) / 4) * 4;
}
inline __host__ __device__ long mailbox_words(int T, int K) {
    return mailbox_miss_offset(T) + 4L * T * K;
}

struct PagerParams {
    const void *ids;
    int ids64, T, K, E, cap, mode, count_forward, single_group;
    // state (device)
    int32_t *s2e;
    int64_t *tick;
    int32_t *emap;
    int64_t *hdr;  // [0] clock, [1..4] forward, miss, hits, evict
    // outputs (device)
    int32_t *slots;      // [T*K]
    int32_t *grp_start;  // [T+1]
    int32_t *grp_nu;     // [T]
    int32_t *u_slot;     // [T*K]       per group at pair offset p0
    int32_t *u_off;      // [T*K + T]   per group at p0 + g (n_u + 1 entries, relative to p0)
    int32_t *u_pairs;    // [T*K]       pair ids grouped by unique expert
    // mailbox (device alias of mapped host memory)
    int32_t *mb;
};

size_t pager_smem_bytes(int E, int cap);
int launch_pager(const PagerParams &p, cudaStream_t stream);

}  // namespace wisp
