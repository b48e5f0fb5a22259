// Persistent, cooperative forward kernel (pager + expert compute in one launch).
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include "decode.cuh"
#include "pager.cuh"

namespace wisp {

// Grid-barrier words (device, per layer): [0] arrivals, [1] generation,
// [2] abort flag, [3] sticky kernel status (first error wins; the host clears it).
enum { kBarArrive = 0, kBarGen = 1, kBarAbort = 2, kBarStatus = 3, kBarWords = 4 };

struct ForwardParams {
    PagerParams pg;                 // block 0 runs the pager with these
    GroupCompute gc;                // x, w13, w2, topk_w, act, y, out, counters, K, H, I
    const uint32_t *slot_ready;     // [cap] generation landed in each slot (copy-stream writes)
    unsigned int *bar;              // [kBarWords]
    unsigned long long *done_word;  // mapped host: (seq << 32) | groups finished
    long long wait_ns;              // limit of any single wait
    int *status_word;               // mapped host: sticky kernel status, cleared by the host
    int publish;                    // block 0 publishes the page-in list (paged mode)
    // dataflow words (device, per layer, kFlowWords): see kFlow* below
    unsigned int *flow;
    int epoch;                      // launch parity: which set of counters this launch uses
    int stages;                     // copy stages per warp (set by launch_forward)
    // the other launch parity's activation buffer, reset here for the next launch
    uint32_t *act_reset;
    long act_reset_words;
    // optional %globaltimer trace (debug): [0..7] block 0 milestones, then 4 words per block
    unsigned long long *trace;
};

// Dataflow words: [kFlowPagerDone] sequence number of the call whose pager
// outputs are complete; [kFlowSpecRead + e] blocks done reading the pre-call
// expert map.  e is the launch parity; a launch zeroes the other one, which
// the next launch uses.  (Gate-up -> down ordering needs no words: a down
// unit polls the activation rows themselves, see kActEmpty.)
constexpr int kFlowPagerDone = 0;
constexpr int kFlowSpecRead = 1;
constexpr int kFlowWords = 8;

int launch_forward(const ForwardParams &p, int max_tokens_per_group, cudaStream_t stream);

}  // namespace wisp
