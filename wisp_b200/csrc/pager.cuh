// Device pager (K1) interface shared by the runtime and the forward kernels.
#pragma once
#include <stddef.h>
#include <stdint.h>

#include <cuda_runtime.h>

namespace wisp {

// Mailbox (mapped pinned host memory, int32 words) written by the pager; the
// host hands each forward a mailbox slot that no unfinished page-in task still
// reads, so the pager never overwrites a mailbox under the reader:
//   [0] status  [1] groups G  [2] misses  [3] failing group  [4] sum of unique experts
//   [5] forward-kernel status (slot 0 only)  [6] reserved  [7] sequence number (written last)
//   [kMbUnique ...]            32 words: bitmap of the forward's unique experts
//   [kMbHeader ...]            group first tokens, G+1 entries (last = T)
//   [kMbHeader + T + 1 ...]    unique experts per group, G entries
//   [mailbox_miss_offset(T)..] page-in records of kMbRec words:
//                              {expert, slot, group, wait_group, generation, 0, 0, 0}
constexpr int kMbUnique = 8;
constexpr int kMbHeader = kMbUnique + 32;
constexpr int kMbRec = 8;
inline __host__ __device__ long mailbox_miss_offset(int T) {
    return ((kMbHeader + 2L * T + 1 + 7) / 8) * 8;
}
inline __host__ __device__ long mailbox_words(int T, int K) {
    return mailbox_miss_offset(T) + (long)kMbRec * T * K;
}

// Device header words written by the pager (read by the forward kernel).
enum { kHdrStatus = 0, kHdrGroups = 1, kHdrMisses = 2, kHdrUnique = 3, kHdrWords = 8 };

struct PagerParams {
    const void *ids;
    int ids64, T, K, E, cap, mode, count_forward, single_group;
    uint32_t seq;  // forward sequence number published in the mailbox
    // state (device)
    int32_t *s2e;
    int64_t *tick;
    int32_t *emap;
    int64_t *hdr;        // [0] clock, [1..4] forward, miss, hits, evict; [5] groups, [6] unique experts (telemetry)
    uint32_t *slot_gen;  // [cap] page-in generation of each slot
    uint32_t *last_unique;  // [E / 32] bitmap: unique experts of the last paged forward (or nullptr)
    // outputs (device)
    int32_t *slots;      // [T*K]
    int32_t *grp_start;  // [T+1]
    int32_t *grp_nu;     // [T]
    int32_t *grp_nhit;   // [T]         experts resident before the group (first in its unique list)
    int32_t *u_slot;     // [T*K]       per group at pair offset p0: hits (ascending id), then misses in page-in order
    int32_t *u_gen;      // [T*K]       slot generation each unique expert waits for (0: none)
    int32_t *u_off;      // [T*K + T]   per group at p0 + g (n_u + 1 entries, relative to p0)
    int32_t *u_pairs;    // [T*K]       pair ids grouped by unique expert
    int32_t *dev_hdr;    // [kHdrWords]
    // mailbox (device alias of mapped host memory)
    int32_t *mb;
};

size_t pager_smem_bytes(int E, int cap, int T, int K);
int launch_pager(const PagerParams &p, cudaStream_t stream);

// Speculative page-in of predicted experts (the reference's prefetch_async,
// fused_moe.py:360-433) on the layer's state; one CTA.  `out` (mapped host
// memory): [0] status, [1] experts to load, then kMbRec words per load
// {expert, slot, generation, 0...}.
struct PrefetchParams {
    const int32_t *pred;          // [n] predicted ids, in the order the caller iterates its set
    int n, E, cap;
    int32_t *s2e;
    int64_t *tick;
    int32_t *emap;
    int64_t *hdr;                 // [0] clock, [4] evictions
    uint32_t *slot_gen;
    const uint32_t *last_unique;  // [E / 32] the layer's last forward's unique experts
    int32_t *out;
};
int launch_prefetch(const PrefetchParams &p, cudaStream_t stream);
// The pager is run by one whole CTA of kPagerThreads threads (pager_body.cuh).
constexpr int kPagerThreads = 256;

}  // namespace wisp
