// Prefill (large token groups) expert compute on tcgen05 tensor cores.
#pragma once
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace wisp {

// One token group whose experts are resident in their slots.
struct PrefillGroup {
    const __nv_bfloat16 *x;         // [T][H] hidden states
    const __nv_bfloat16 *w13;       // slot scratch [slots][2I][H]
    const __nv_bfloat16 *w2;        // slot scratch [slots][H][I]
    int slots;                      // slot count (tensor-map extent)
    const int32_t *u_off;           // [nu + 1] group-local offsets into u_pairs
    const int32_t *u_pairs;         // [npairs] absolute pair index t * K + k, expert-major
    const int32_t *u_slot;          // [nu]
    const int32_t *nu_dev;          // experts in the group (device word written by the pager)
    const int32_t *pager_status;    // pager status (device); nullptr when the host checked it
    const int32_t *u_gen;           // [nu] page-in generation each expert's slot must reach (0: resident
                                    // before the call), or nullptr: the slots are ready at launch
    const uint32_t *slot_ready;     // [slots] generation landed in each slot (written by the copy stream)
    int nu, npairs;                 // nu: upper bound of *nu_dev (grid sizes)
    int t0, t1, K, H, I;
    const float *topk_w;            // [T * K]
    __nv_bfloat16 *x_perm;          // [perm_rows][H] workspace
    __nv_bfloat16 *act_perm;        // [perm_rows][I] workspace
    int perm_rows;                  // rows of the two workspaces (>= npairs)
    __nv_bfloat16 *y;               // [T * K][H]
    __nv_bfloat16 *out;             // [T][H]
    int *status;                    // sticky status word
    long long wait_ns;
    unsigned long long *trace;      // debug milestones (weight-stationary kernel), or nullptr
};

// The tensor-core path covers hidden % 256 == 0 and inter % 128 == 0.
bool prefill_shapes_supported(int H, int I);

// Launches gather, gate-up GEMM, down GEMM and combine (4 kernels) on `stream`.
constexpr int kPrefillKernelsPerGroup = 4;
int launch_prefill_group(const PrefillGroup &p, cudaStream_t stream);

// Weight-stationary tensor-core path for decode batches (few tokens per
// expert, at most kBatchMaxPairs pairs per group).
constexpr int kBatchTokens = 32;     // token rows per tile (the MMA's N)
constexpr int kBatchMaxPairs = 512;  // pairs of one call (or group) on this path
// Per-token-block counters, then a gathered-rows counter, the tile
// scheduler's counter and an abort word.
constexpr long kBatchReadyWords = kBatchMaxPairs + (kBatchMaxPairs + kBatchTokens - 1) / kBatchTokens + 3;

// Per-launch counters of the path, two halves by launch parity: a launch
// uses one half and zeroes the other for the next launch.
__host__ __device__ inline int batch_done_words(int H) { return kBatchMaxPairs * (H / 256) * 4; }
struct BatchCounters {
    uint32_t *ready, *ready_next;  // kBatchReadyWords each: gate-up warps done per token block
    uint32_t *done, *done_next;    // batch_done_words(H) each: down rows stored per token
};

// A group whose expert lists come from the pager (paged layers): gather and
// one persistent launch that runs gate-up, down and the routing-order
// combine of the group's tokens (2 kernels).
constexpr int kBatchKernelsPerGroup = 2;
int launch_batch_group(const PrefillGroup &p, const BatchCounters &c, cudaStream_t stream);

// A whole call of a resident layer in one launch: the persistent kernel
// routes the pairs itself (counting sort by expert in every CTA, ascending
// pair order within an expert), gathers the hidden rows its tiles read,
// counts the forward in the pager counters (forward, groups, unique experts),
// then runs gate-up, down and the combine.  A routed id outside [0, E) stops
// the call before any counter changes and records WISP_ERR_BAD_EXPERT in the
// sticky word and in *dev_status; out is left alone.
struct BatchRoute {
    const void *ids;
    int ids64, E, count_forward;
    const int32_t *emap;   // [E] slot of each expert
    int64_t *hdr;          // pager counters: [1] forward, [5] groups, [6] unique experts
    int32_t *dev_status;   // this call's routing status (device)
};
constexpr int kBatchKernelsResident = 1;
int launch_batch_resident(const PrefillGroup &p, const BatchRoute &r, const BatchCounters &c, cudaStream_t stream);

// A whole call of a resident layer on the token-major GEMMs: one cooperative
// kernel writes the group lists the GEMMs read (the pairs sorted by expert,
// experts ascending; each expert's slot from the map; the count into *nu and
// the group header words), gathers the pairs' token rows into X_perm and
// counts the forward as the weight-stationary path does; then gate-up, down
// and combine run on them.  p.u_off / u_pairs / u_slot / nu_dev must be the
// addresses the routing kernel writes (`lists`); r.dev_status is the group
// header (status word first).  `cnt` / `cnt_next`: the routing counters of
// this launch and of the next (2 E + 1 words each, two halves by launch
// parity); `bar`: two words of the kernel's grid barrier.  A routed id
// outside [0, E) leaves the lists alone, records WISP_ERR_BAD_EXPERT in the
// header and the sticky word, and the other kernels of the call then do
// nothing.
struct PrefillLists {
    int32_t *u_off, *u_pairs, *u_slot, *nu;
    int32_t *cnt, *cnt_next;
    uint32_t *bar;
};
constexpr int kPrefillKernelsResident = kPrefillKernelsPerGroup;
int launch_prefill_resident(const PrefillGroup &p, const BatchRoute &r, const PrefillLists &lists,
                            cudaStream_t stream);

}  // namespace wisp
