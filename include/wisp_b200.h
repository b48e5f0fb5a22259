/*
 * wisp_b200.h - C ABI of the B200 paged fused-MoE layer.
 *
 * One opaque handle per MoE layer holds what the reference keeps in a
 * per-layer ``WispMoEState`` (src/wisp/integrations/vllm/fused_moe.py:126-236):
 * the pinned host masters of the expert weights (caller-owned), the HBM slot
 * scratch, the expert->slot map, the LRU state and the counters.  The LRU
 * pager runs on the device, page-in runs on copy-engine streams, expert
 * compute runs in hand-written sm_100a kernels.
 *
 * Conventions
 *   - every function returns a status (WISP_OK == 0); on failure
 *     wisp_last_error() gives a message for the calling thread;
 *   - ``stream`` is a cudaStream_t passed as void* (NULL = legacy default
 *     stream); x / topk_* / out pointers are device pointers;
 *   - expert weights are bf16: w13 [E][2I][H] (gate rows then up rows), w2
 *     [E][H][I], like vLLM's UnquantizedFusedMoEMethod.create_weights.
 */
#ifndef WISP_B200_H
#define WISP_B200_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define WISP_API __attribute__((visibility("default")))
#else
#define WISP_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

typedef struct wisp_layer wisp_layer;

enum wisp_status {
    WISP_OK = 0,
    WISP_ERR_INVALID = 1,      /* bad argument / shape / unpinned host memory */
    WISP_ERR_OVERFLOW = 2,     /* one call's unique experts exceed the cap ("sub-batch" error) */
    WISP_ERR_BAD_EXPERT = 3,   /* routed expert id outside [0, E) */
    WISP_ERR_CUDA = 4,         /* a CUDA runtime call failed */
    WISP_ERR_TIMEOUT = 5,      /* a bounded device or host wait ran out */
    WISP_ERR_NOMEM = 6,        /* device or pinned allocation failed */
    WISP_ERR_UNSUPPORTED = 7   /* shape/mode not supported by the compute kernels */
};

enum wisp_mode { WISP_MODE_PAGED = 0, WISP_MODE_RESIDENT = 1 };

/* Library version string and the message of this thread's last failure. */
WISP_API const char *wisp_version(void);
WISP_API const char *wisp_last_error(void);

/*
 * Create a layer.  Replaces WispMoEState.__init__ (fused_moe.py:161-236):
 * scratch [cap][w13_expert_bytes] and [cap][w2_expert_bytes] in HBM,
 * expert_map[E] = -1, slot_to_expert[cap] = -1, lru_tick[cap] = 0, clock 0.
 * host_w13 / host_w2 are the pinned host masters ([E][bytes] each); they
 * must stay alive and pinned for the layer's lifetime.  hidden / inter give
 * the bf16 compute shape (0, 0 for a paging-only layer).
 */
WISP_API int wisp_layer_create(int32_t num_experts, int32_t cap_experts, int32_t hidden,
                      int32_t inter, int64_t w13_expert_bytes, int64_t w2_expert_bytes,
                      const void *host_w13, const void *host_w2, int32_t device,
                      int32_t mode, wisp_layer **out);
WISP_API int wisp_layer_destroy(wisp_layer *layer);

/*
 * Create a block-quantised FP8 layer: the reference's WispMoEStateFP8
 * (fused_moe_fp8.py:61-145), which pages (weight, scale) pairs.  Host masters
 * (pinned, caller-owned): w13 [E][2I][H] and w2 [E][H][I] float8_e4m3fn, and
 * their per-128x128-block fp32 scales s13 [E][2I/128][H/128] and s2
 * [E][H/128][I/128] (vLLM's w*_weight_scale_inv).  block_n = block_k = 128;
 * hidden and inter multiples of 128.  Paging, the pager and every other entry
 * point behave as for a bf16 layer; the compute is W8A8 with per-token-group
 * activation quantisation (the arithmetic of vLLM's block-FP8 fused_experts)
 * on the CUDA cores, through the host-synchronous forward at every call size.
 */
WISP_API int wisp_layer_create_fp8(int32_t num_experts, int32_t cap_experts, int32_t hidden, int32_t inter,
                                   int32_t block_n, int32_t block_k, const void *host_w13, const void *host_w2,
                                   const void *host_s13, const void *host_s2, int32_t device, int32_t mode,
                                   wisp_layer **out);

/*
 * Paged MoE forward of ``num_tokens`` rows, enqueued on ``stream`` (the call
 * returns before the work runs; see wisp_layer_sync for errors).  Replaces the pager + compute of
 * _wisp_forward_cuda_paged (fused_moe.py:1017, 1102-1168) and vLLM
 * fused_experts with expert_map (called at fused_moe.py:1106-1118, 1155-1167):
 * first-fit token sub-batching, one LRU step per group (bit-exact with the
 * reference's ensure_resident), page-in of the misses, gate-up GEMM + SiLU-mul,
 * down GEMM x routing weight, routing-order combine.
 *   x [T][H] bf16, topk_weights [T][k] fp32, topk_ids [T][k] int32 or int64
 *   (ids_int64 != 0), out [T][H] bf16.
 * Returns WISP_ERR_OVERFLOW when a single token routes to more unique
 * experts than the cap (the reference raises RuntimeError "...sub-batch..."),
 * WISP_ERR_INVALID for a resident layer before wisp_prime_identity.
 */
WISP_API int wisp_moe_forward(wisp_layer *layer, const void *x, const float *topk_weights,
                     const void *topk_ids, int32_t ids_int64, int32_t num_tokens,
                     int32_t top_k, void *out, void *stream);

/*
 * Router for callers that hold router logits: per token, fp32 softmax over
 * the num_experts logits (fp32, or bf16 when logits_bf16), the top_k largest
 * probabilities in descending order (ties to the lower expert id) and, when
 * renormalize, the weights divided by their sum -- the routing the reference's
 * paged forward takes from vLLM's select_experts (fused_moe.py:1054-1076).
 * topk_weights [T][k] fp32, topk_ids [T][k] int32; asynchronous on `stream`.
 * num_experts <= 1024, top_k <= 32.
 */
WISP_API int wisp_route_topk(const void *logits, int32_t logits_bf16, int32_t num_tokens, int32_t num_experts,
                             int32_t top_k, int32_t renormalize, float *topk_weights, int32_t *topk_ids,
                             void *stream);

/*
 * One LRU admission step for an arbitrary id list, with page-in, finished
 * before returning.  Replaces WispMoEState.ensure_resident
 * (fused_moe.py:264-358).
 */
WISP_API int wisp_ensure_resident(wisp_layer *layer, const void *ids, int32_t ids_int64, int32_t n,
                         void *stream);

/*
 * Pager side of one forward without the expert compute: first-fit groups, one
 * LRU step per group, page-in, finished before returning; writes the slot each
 * (token, k) read to slots_out (host, [T][k]; may be NULL).  The test and replay
 * hook for the bookkeeping of _wisp_forward_cuda_paged (fused_moe.py:1017,
 * 1102-1168).
 */
WISP_API int wisp_pager_step(wisp_layer *layer, const void *topk_ids, int32_t ids_int64,
                             int32_t num_tokens, int32_t top_k, int32_t *slots_out, void *stream);

/*
 * Speculative page-in of predicted experts: the reference's
 * WispMoEState.prefetch_async (fused_moe.py:360-433), bit-exact.  predicted
 * (host, n <= E ids) in the order the caller iterates its predicted set.
 * Experts with no slot are loaded, in that order; victims are taken by LRU
 * (tick, slot) among slots whose expert is neither predicted nor in the
 * layer's last forward's unique set; a prediction larger than the free slots
 * plus those victims is loaded in part; the clock moves only when something
 * loads; evictions count, misses and hits do not.  The state changes and the
 * page-ins run on the layer's copy stream after its last forward, and its
 * next forward waits for them.  Returns once the copies are issued.
 */
WISP_API int wisp_prefetch_async(wisp_layer *layer, const int32_t *predicted, int32_t n, void *stream);

/* Resident mode: identity map and full copy.  fused_moe.py:242-258 (cap == E). */
WISP_API int wisp_prime_identity(wisp_layer *layer, void *stream);

/* Hot resize of the slot scratch, clamped to [2, E].  fused_moe.py:439-490. */
WISP_API int wisp_resize_cap(wisp_layer *layer, int32_t new_cap, void *stream);

/*
 * Read back the pager state (synchronises the device).  Any pointer may be
 * NULL.  stats4 = {forward, miss, hits, evict} (fused_moe.py:211-221).
 */
WISP_API int wisp_get_state(wisp_layer *layer, int32_t *slot_to_expert, int64_t *lru_tick,
                   int64_t *clock, int64_t *stats4, int32_t *expert_map, int32_t *cap);

/* Overwrite the four counters (snapshot_expert_stats reset, fused_moe.py:579-593). */
WISP_API int wisp_set_stats(wisp_layer *layer, const int64_t *stats4);

/* Device addresses of the slot scratch and expert map (for zero-copy views). */
WISP_API int wisp_layer_buffers(wisp_layer *layer, void **scratch_w13, void **scratch_w2,
                       void **expert_map);

/* Device addresses of an FP8 layer's slot scales (scratch_s13, scratch_s2). */
WISP_API int wisp_layer_scale_buffers(wisp_layer *layer, void **scratch_s13, void **scratch_s2);

/*
 * Cumulative telemetry (synchronises the device): {groups run, misses,
 * page-in bytes, unique experts read summed over groups}.
 */
WISP_API int wisp_get_telemetry(wisp_layer *layer, int64_t *out4);

/*
 * The unique expert ids, ascending, of this layer's last paged forward
 * (synchronises the device): the reference's WispMoEState.last_unique_experts
 * (fused_moe.py:1170-1176), which snapshot_expert_stats reports as the working
 * set (:579-593) and prefetch_async keeps out of its victims (:360-433).  A
 * resident forward leaves it unchanged, as the reference's does.  Writes at
 * most max_ids ids; *n_out = the number of unique experts.
 */
WISP_API int wisp_get_last_unique_experts(wisp_layer *layer, int32_t *ids_out, int32_t max_ids,
                                          int32_t *n_out);

/*
 * Number of CUDA kernels this layer has launched so far, on every path (one
 * per asynchronous forward; pager plus two per token group on the synchronous
 * path).  No counterpart in the reference; used to account for launches.
 */
WISP_API int wisp_get_launch_count(wisp_layer *layer, int64_t *out);

/*
 * Wait until every forward issued on this layer has finished (kernels and
 * page-ins) and return the first error any of them hit since the last check
 * (WISP_OK if none).  wisp_moe_forward returns before its work runs; a
 * device-side failure (a routed id outside [0, E), a bounded wait that ran
 * out) is reported by the next wisp_moe_forward or wisp_layer_sync.  After a
 * timeout a paged layer restarts cold (no slot resident; clock and counters
 * kept); a resident layer keeps its slots.
 */
WISP_API int wisp_layer_sync(wisp_layer *layer);

/*
 * Size the layer's per-call workspace for calls of up to num_tokens tokens at
 * top_k now, at set-up, instead of at the first call that needs it (growing
 * it waits for the device and reallocates: a stall in the middle of serving;
 * an expert-parallel owner, whose call size varies with what it receives,
 * reserves the largest receive).  No effect when the workspace is already
 * that large.  (No reference counterpart: the reference allocates per call.)
 */
WISP_API int wisp_layer_reserve(wisp_layer *layer, int32_t num_tokens, int32_t top_k);

/*
 * Cross-layer co-activation table and prefetch predictor (host C++), the
 * reference's CooccurTable / predict_layer (src/wisp/oracle/cooccur.py:44-292)
 * with the same counts, scores (double, the reference's expression and
 * accumulation order) and ranking (score descending, id ascending).  Layers
 * and their experts are passed in CSR form: layers[i] with experts
 * experts[offsets[i] .. offsets[i+1]), in the order the caller's dict holds
 * them.  Export lists pairs [L_src, e_src, L_dst, e_dst, n] (n > 0) and
 * marginals [L, e, n] in first-seen order (the reference's JSON schema).
 */
typedef struct wisp_cooccur wisp_cooccur;
WISP_API int wisp_cooccur_create(wisp_cooccur **out);
WISP_API int wisp_cooccur_destroy(wisp_cooccur *table);
WISP_API int wisp_cooccur_observe_step(wisp_cooccur *table, int32_t n_layers, const int32_t *layers,
                                       const int32_t *offsets, const int32_t *experts);
WISP_API int wisp_cooccur_predict(const wisp_cooccur *table, int32_t n_seen, const int32_t *layers,
                                  const int32_t *offsets, const int32_t *experts, int32_t target_layer, int32_t k,
                                  int32_t normalize, double decay, int32_t only_prev_layer, int32_t *out_ids,
                                  int32_t *n_out);
WISP_API int wisp_cooccur_set_pair(wisp_cooccur *table, int32_t l_src, int32_t e_src, int32_t l_dst, int32_t e_dst,
                                   int64_t n);
WISP_API int wisp_cooccur_set_marginal(wisp_cooccur *table, int32_t l, int32_t e, int64_t n);
WISP_API int wisp_cooccur_set_steps(wisp_cooccur *table, int64_t steps);
WISP_API int wisp_cooccur_sizes(const wisp_cooccur *table, int64_t *n_sources, int64_t *n_pairs,
                                int64_t *n_marginals, int64_t *steps);
WISP_API int wisp_cooccur_export(const wisp_cooccur *table, int64_t *pairs, int64_t max_pairs, int64_t *n_pairs,
                                 int64_t *marginals, int64_t max_marginals, int64_t *n_marginals);

/*
 * Tunables: WISP_CFG_ASYNC (1: single-launch forward with asynchronous
 * page-in, the default of resident layers; 0: host-synchronous path, the
 * default of paged layers -- a paged single-launch forward waits inside the
 * kernel for copies a host thread issues after the launch, so the caller must
 * queue no other device work while it pages in, or the copies can be held
 * behind that work until the wait limit), WISP_CFG_WAIT_NS (limit of
 * one device-side wait, default 10 s), WISP_CFG_DROP_PAGEINS (test fault: the
 * host silently skips the next n page-ins of this layer),
 * WISP_CFG_TRACE_BUFFER (debug: device address of a uint64 buffer that
 * the one-launch forward kernel (8 + 4096 + 16 * warps of the grid words,
 * at most 32520 on 148 SMs) and the weight-stationary tensor-core kernel
 * (8 + 8 * grid words) fill with %globaltimer milestones; 0 = off), WISP_CFG_TC_MIN_PAIRS (calls of at least this many
 * (token, k) pairs run their expert compute on the tcgen05 tensor cores --
 * weight-stationary tiles up to 512 pairs, token-major GEMMs above -- where
 * hidden % 256 == 0 and inter % 128 == 0; smaller calls on the CUDA-core
 * decode kernels.  The choice depends on the call size only, so outputs stay
 * byte-identical across caps and modes; default: the smallest call whose
 * weight-stationary tiles, (I / 128 + H / 256) per pair at most, could fill
 * the GPU twice over -- 22 pairs at Qwen3-30B-A3B shapes on 148 SMs;
 * capped at 513),
 * WISP_CFG_COMPUTE_CLASS (0: by call size as above, the default; 1: the
 * CUDA-core kernels at any size; 2: the tensor cores at any size.  The two
 * tensor-core paths give identical bytes, the CUDA-core kernels differ in
 * the fp32 accumulation order: an expert-parallel owner computes each
 * source's rows in the class a one-GPU call of that source's size would
 * use).
 */
enum wisp_config_key {
    WISP_CFG_ASYNC = 1,
    WISP_CFG_WAIT_NS = 2,
    WISP_CFG_DROP_PAGEINS = 4,
    WISP_CFG_TRACE_BUFFER = 5,
    WISP_CFG_TC_MIN_PAIRS = 6,
    WISP_CFG_COMPUTE_CLASS = 7
};
WISP_API int wisp_layer_config(wisp_layer *layer, int32_t key, int64_t value);
/* Current value of a tunable (WISP_CFG_ASYNC, _WAIT_NS, _TC_MIN_PAIRS,
 * _COMPUTE_CLASS); no counterpart in the reference. */
WISP_API int wisp_layer_query(wisp_layer *layer, int32_t key, int64_t *value);

/*
 * Expert compute from slot scratch that allocates nothing (this entry point
 * has no counterpart in the reference, which always lets vLLM allocate).
 * For callers that may not call cudaMalloc: plug-ins inside a serving engine
 * that has reserved the free HBM for its KV cache and hands out only its own
 * buffers, or decode loops that cannot take cudaMalloc's implicit device
 * synchronisation.  Runs the decode kernels of wisp_moe_forward on given
 * slots: x [T][H] bf16, scratch_w13 [num_slots][2I][H] / scratch_w2
 * [num_slots][H][I] bf16, pair_slots [T][k] int32 (the slot each (t, k)
 * reads; a slot outside [0, num_slots) contributes zero), topk_weights
 * [T][k] fp32, out [T][H] bf16.  Intermediates live in one static device
 * array of about 6.3 MB per GPU, held until exit: T*k <= 128, hidden <= 8192,
 * inter <= 16384; larger sizes return WISP_ERR_INVALID.  Calls share that
 * array, so calls that overlap on the GPU race.  CUDA loads device code, and
 * with it this array, onto a GPU lazily: the array takes its device memory at
 * the first call on that device, not when the library is loaded.  A call with
 * num_tokens == 0 (the other arguments except device are then ignored) does
 * only that set-up -- places the array and the kernels' code on `device` and
 * resolves the array's address (cudaGetSymbolAddress) with that device
 * current -- and computes nothing; make it at start-up, before reserving the
 * free HBM and before any stream capture.  From then on the GPU holds the
 * array until the process exits.
 */
WISP_API int wisp_expert_compute_noalloc(int32_t device, const void *x, const void *scratch_w13,
                                         const void *scratch_w2, int32_t num_slots,
                                         const int32_t *pair_slots, const float *topk_weights,
                                         int32_t num_tokens, int32_t top_k, int32_t hidden,
                                         int32_t inter, void *out, void *stream);

/*
 * Expert parallelism (no counterpart in the reference, which runs one GPU per
 * layer).  Rank r of `world` owns experts [r * experts_per_rank,
 * (r + 1) * experts_per_rank) and pages only those.  The (token, k) pairs go
 * to their owners over peer memory (NVLink / NVSwitch): each rank's group
 * holds one region with the same layout on every rank, mapped into every
 * peer through CUDA IPC, and the kernels below store rows straight into the
 * peer's region (plain stores; no collective library on the data path).
 * Per layer forward every rank calls, in this order:
 *   wisp_ep_dispatch   route the call's pairs and store their rows and
 *                      records into the owners' receive segments;
 *   wisp_ep_receive    wait for every source, compact the received rows
 *                      (by run of same-class sources, by local expert
 *                      within a run) into the group's x_recv / ids_recv /
 *                      w_recv and return the counts to the host;
 *   the owner's own wisp_moe_forward on x_recv[0:R] (top_k 1, local ids)
 *   into y_recv[0:R];
 *   wisp_ep_return     store each weighted row back into its source;
 *   wisp_ep_combine    wait for every owner and write out[t] = the
 *                      routing-order sum of the token's k rows (the one-GPU
 *                      combine, so the output is byte-identical to a one-GPU
 *                      layer whose compute takes the same kernels).
 * Each dispatch starts a new epoch; every wait is bounded (default 10 s,
 * wisp_ep_group_config) and a wait that runs out is reported, never hangs.
 */
typedef struct wisp_ep_group wisp_ep_group;

/* This rank's exchange buffers for calls of at most max_pairs (token, k)
 * pairs per rank and hidden size `hidden` (a multiple of 8). */
WISP_API int wisp_ep_group_create(int32_t rank, int32_t world, int32_t device, int32_t max_pairs,
                                  int32_t hidden, wisp_ep_group **out);
/* The 64-byte CUDA IPC handle of this rank's region (to all-gather). */
WISP_API int wisp_ep_group_ipc_handle(wisp_ep_group *group, void *handle_out);
/* Map every peer's region: handles = world consecutive 64-byte handles, by rank. */
WISP_API int wisp_ep_group_connect(wisp_ep_group *group, const void *handles);
/* Ranks emulated in one process on one device: groups[r] is rank r's group. */
WISP_API int wisp_ep_group_connect_local(wisp_ep_group *group, wisp_ep_group *const *groups);
WISP_API int wisp_ep_group_destroy(wisp_ep_group *group);
/* Device addresses of the owner-side buffers: x_recv [world*max_pairs][H]
 * bf16, ids_recv int32, w_recv fp32, y_recv [world*max_pairs][H] bf16. */
WISP_API int wisp_ep_group_buffers(wisp_ep_group *group, void **x_recv, void **ids_recv, void **w_recv,
                                   void **y_recv);
/* Limit of one device-side wait of this group's kernels (nanoseconds). */
WISP_API int wisp_ep_group_config(wisp_ep_group *group, int64_t wait_ns);
/* x [T][H] bf16, topk_ids [T][k] int32 (int64 when ids_int64), topk_weights
 * [T][k] fp32; asynchronous on `stream`.  An id outside [0, world *
 * experts_per_rank) makes every rank's wisp_ep_receive fail alike. */
WISP_API int wisp_ep_dispatch(wisp_ep_group *group, const void *x, const void *topk_ids, int32_t ids_int64,
                              const float *topk_weights, int32_t num_tokens, int32_t top_k,
                              int32_t experts_per_rank, void *stream);
/* Synchronous: returns when the received rows are compacted.  A run is a
 * maximal range of consecutive sources (rank order, sources with rows) of one
 * compute class -- sources of at least class_min_pairs (token, k) pairs form
 * one class (0: a single class); rows keep their run and are ordered by local
 * expert within it, stably.  counts_out / src_pairs_out (host, [world], may
 * be NULL): rows from each source and each source's pair count; total_out:
 * rows received. */
WISP_API int wisp_ep_receive(wisp_ep_group *group, int32_t class_min_pairs, void *stream, int32_t *counts_out,
                             int32_t *src_pairs_out, int32_t *total_out);
/* Store y_recv[0:R] (R of the last receive) back into the sources. */
WISP_API int wisp_ep_return(wisp_ep_group *group, void *stream);
/* out [T][H] bf16 = routing-order sum of this rank's returned rows. */
WISP_API int wisp_ep_combine(wisp_ep_group *group, int32_t num_tokens, int32_t top_k, void *out, void *stream);
/* Wait for the device and report (then clear) a failure of the group's kernels. */
WISP_API int wisp_ep_sync(wisp_ep_group *group);

#ifdef __cplusplus
}
#endif

#endif /* WISP_B200_H */
