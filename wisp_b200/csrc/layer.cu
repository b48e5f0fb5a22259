// Per-layer runtime behind the C ABI (include/wisp_b200.h).
//
// A wisp_layer is the B200 counterpart of the reference's WispMoEState
// (src/wisp/integrations/vllm/fused_moe.py:126-490): slot scratch in HBM,
// the expert map and LRU state in device memory (owned by the device pager),
// a copy-engine stream for page-in from the caller's pinned host masters,
// and the compute kernels.
//
// Forward, one-launch path (default for resident layers; a paged layer opts
// in with WISP_CFG_ASYNC, when top_k <= cap so the working-set overflow of
// fused_moe.py:313-327 cannot happen):
//   * one cooperative launch of the persistent forward kernel (forward.cu)
//     on the caller's stream: pager, then per group gate-up / down / combine;
//     the host does not wait;
//   * the per-device page-in engine (a host thread) picks up the call's
//     page-in list from the mailbox the pager fills (mapped pinned memory,
//     guarded by a sequence number), and for each miss, once the kernel has
//     published that the last earlier group reading the victim slot is done,
//     issues the two H2D copies on the layer's copy stream followed by a
//     stream memory write of the slot's generation flag, which is what the
//     kernel waits on before reading the slot.  (The kernel waits on work
//     issued after it; see wisp_layer_create for why paged layers do not
//     take this path by default.)
// Forward, synchronous path (default for paged layers; top_k > cap): the
// pager kernel runs alone, the host reads the mailbox, issues the page-ins of
// each group with event ordering and launches the per-group decode kernels.
// Both paths run the same warp arithmetic (moe_body.cuh), so their outputs are
// byte-identical.
#include <cuda.h>

#include <algorithm>
#include <atomic>
#include <cstdlib>
#include <chrono>
#include <condition_variable>
#include <deque>
#include <memory>
#include <mutex>
#include <string>
#include <thread>
#include <vector>

#include "common.cuh"
#include "decode.cuh"
#include "forward.cuh"
#include "fp8.cuh"
#include "pager.cuh"
#include "prefill.cuh"

namespace wisp {

static thread_local std::string g_last_error;
void set_error(const std::string &msg) { g_last_error = msg; }

namespace {
std::atomic<int> g_pdl_state[64];  // 0 untried / accepted, 1 refused
int pdl_env() {
    // opt-in: no gain was measurable on one GPU, and expert-parallel runs with
    // it on measured their timed region at half the end-to-end rate
    static const int v = std::getenv("WISP_PDL") ? 1 : 0;
    return v;
}
}  // namespace
bool pdl_enabled(int dev) { return pdl_env() && dev >= 0 && dev < 64 && g_pdl_state[dev].load() == 0; }
void pdl_refused(int dev) {
    if (dev >= 0 && dev < 64) g_pdl_state[dev].store(1);
}

namespace {

struct DeviceGuard {
    int prev = -1;
    explicit DeviceGuard(int dev) {
        if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
        if (prev != dev) cudaSetDevice(dev);
    }
    ~DeviceGuard() {
        int cur = -1;
        if (prev >= 0 && cudaGetDevice(&cur) == cudaSuccess && cur != prev) cudaSetDevice(prev);
    }
};

int fail(int code, const std::string &msg) {
    set_error(msg);
    return code;
}

bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// cuStreamWriteValue32 through the runtime's driver entry point (no link
// against libcuda, so the library loads on machines without a driver).
typedef CUresult (*WriteValue32Fn)(CUstream, CUdeviceptr, cuuint32_t, unsigned int);
WriteValue32Fn g_write32 = nullptr;
std::once_flag g_write32_once;

void init_write32() {
    void *fn = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPoint("cuStreamWriteValue32", &fn, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess && fn)
        g_write32 = reinterpret_cast<WriteValue32Fn>(fn);
    else
        cudaGetLastError();
}

constexpr long long kDefaultWaitNs = 10LL * 1000 * 1000 * 1000;
// Calls of T * k pairs in [tc_min_pairs, kPrefillMinPairs) run on the
// weight-stationary tensor-core path, larger ones on the token-major GEMMs,
// smaller ones on the CUDA-core decode kernels.
constexpr int kPrefillMinPairs = kBatchMaxPairs + 1;

// Default tensor-core threshold of a layer: the smallest call whose
// weight-stationary tiles -- I / 128 gate-up + H / 256 down per pair at most
// -- could fill the GPU twice over, so calls of one tile per SM or fewer stay
// on the CUDA-core kernels, which spread an expert over every SM.  It
// depends on the expert shape only (not on E), so an expert-parallel shard
// and a one-GPU layer of the same model choose alike.  (Qwen3-30B-A3B
// shapes on 148 SMs: 22 pairs; measured crossover between 16 and 24.)
int default_tc_min_pairs(int H, int I, int sms) {
    const int per = I / 128 + H / 256;
    if (per <= 0 || sms <= 0) return kPrefillMinPairs;
    return std::min(std::max((2 * sms + per - 1) / per, 1), kPrefillMinPairs);
}
constexpr int kMbRing = 4;

}  // namespace
}  // namespace wisp

using namespace wisp;

struct wisp_layer {
    int dev = 0, E = 0, cap = 0, H = 0, I = 0, mode = WISP_MODE_PAGED;
    int64_t b13 = 0, b2 = 0;
    const char *h13 = nullptr, *h2 = nullptr;
    char *d13 = nullptr, *d2 = nullptr;
    // block-quantised FP8 layers: per-expert fp32 block scales beside the weights
    bool fp8 = false;
    int64_t bs13 = 0, bs2 = 0;
    const char *hs13 = nullptr, *hs2 = nullptr;
    char *ds13 = nullptr, *ds2 = nullptr;
    uint8_t *d_xq = nullptr, *d_aq = nullptr;  // FP8 workspace: quantised tokens and activations
    float *d_xs = nullptr, *d_as = nullptr;
    int32_t *d_s2e = nullptr, *d_emap = nullptr;
    int64_t *d_tick = nullptr, *d_hdr = nullptr;
    uint32_t *d_slot_gen = nullptr, *d_slot_ready = nullptr;
    uint32_t *d_last_unique = nullptr;  // bitmap of the last paged forward's unique experts
    uint32_t h_last_unique[32] = {};    // host copy, valid when the host read the last forward's mailbox
    bool last_unique_host = false;
    int32_t *h_pf = nullptr, *d_pf = nullptr;  // prefetch: predicted ids [E], then status / records (mapped)
    cudaEvent_t ev_pf = nullptr;
    unsigned int *d_bar = nullptr;
    unsigned int *d_flow = nullptr;  // forward-kernel dataflow words (kFlowWords)
    int kparity = 0;                 // parity of the forward-kernel launches
    int64_t launches = 0;            // kernels this layer launched (all paths)
    bool act_dirty = true;           // activation buffers not all kActEmpty (see forward_async)
    // per-call workspace, grown on demand
    int wsT = -1, wsK = 0;
    int32_t *d_slots = nullptr, *d_grp_start = nullptr, *d_grp_nu = nullptr, *d_grp_nhit = nullptr,
            *d_u_slot = nullptr, *d_u_gen = nullptr, *d_u_off = nullptr, *d_u_pairs = nullptr,
            *d_counters = nullptr, *d_dev_hdr = nullptr;
    __nv_bfloat16 *d_act = nullptr, *d_y = nullptr;
    __nv_bfloat16 *d_xperm = nullptr, *d_actperm = nullptr;  // tensor-core paths: rows, expert-major
    uint32_t *d_ready = nullptr;     // weight-stationary path: per-token-block counters, two halves
    uint32_t *d_combined = nullptr;  // weight-stationary path: per-token combine counters, two halves
    int ready_parity = 0;            // the halves the next weight-stationary launch uses
    int32_t *d_route = nullptr;      // resident prefill routing: two halves of 2 E + 1 counters, 2 barrier words
    int route_parity = 0;
    int tc_min_pairs = kPrefillMinPairs;  // calls of at least this many pairs run on the tensor cores
    int compute_class = 0;           // 0: by call size; 1: CUDA-core kernels; 2: tensor cores
    bool primed = false;             // resident layer: every expert copied into its slot
    int32_t *h_mb = nullptr, *d_mb = nullptr;  // kMbRing mailboxes of mb_words words
    long mb_words = 0;
    int mb_next = 0;
    std::atomic<int> mb_busy[4];                // a page-in task still reads this mailbox
    int32_t *h_status = nullptr, *d_status = nullptr;  // sticky forward-kernel status (mapped)
    unsigned long long *h_done = nullptr, *d_done = nullptr;
    uint32_t *h_flag_ring = nullptr;  // pinned sources of flag copies when stream writes are missing
    std::atomic<uint32_t> flag_idx{0};
    cudaStream_t copy_stream = nullptr;
    cudaEvent_t ev_pager = nullptr, ev_copies = nullptr, ev_last = nullptr;
    // resident forwards skip the two event waits when stream order already
    // covers them: the last forward ran on the same stream and no copy was
    // queued since that stream waited for the copies
    cudaStream_t last_stream = nullptr;
    bool last_stream_set = false;
    uint64_t copy_gen = 0, copy_waited = ~0ull;
    std::vector<cudaEvent_t> ev_group, ev_copy;
    uint32_t seq = 0;
    bool async = true;
    long long wait_ns = kDefaultWaitNs;
    unsigned long long *trace = nullptr;  // debug: device buffer for forward-kernel timestamps
    std::atomic<int> drop_pageins{0};
    std::atomic<int> host_status{0};
    std::atomic<int> pending{0};  // page-in tasks queued for this layer
    std::mutex mu;
};

namespace {

constexpr int kFlagRing = 1 << 16;

// ---------------------------------------------------------------------------
// Page-in issue (both paths): two H2D copies, then the slot's generation flag.
// ---------------------------------------------------------------------------
int issue_pagein(wisp_layer *L, int64_t e, int64_t s, uint32_t gen) {
    WISP_CUDA_TRY(cudaMemcpyAsync(L->d13 + s * L->b13, L->h13 + e * L->b13, L->b13,
                                  cudaMemcpyHostToDevice, L->copy_stream));
    WISP_CUDA_TRY(cudaMemcpyAsync(L->d2 + s * L->b2, L->h2 + e * L->b2, L->b2, cudaMemcpyHostToDevice,
                                  L->copy_stream));
    if (L->fp8) {  // the (weight, scale) pairs travel together
        WISP_CUDA_TRY(cudaMemcpyAsync(L->ds13 + s * L->bs13, L->hs13 + e * L->bs13, L->bs13,
                                      cudaMemcpyHostToDevice, L->copy_stream));
        WISP_CUDA_TRY(cudaMemcpyAsync(L->ds2 + s * L->bs2, L->hs2 + e * L->bs2, L->bs2, cudaMemcpyHostToDevice,
                                      L->copy_stream));
    }
    if (g_write32) {
        CUresult r = g_write32(reinterpret_cast<CUstream>(L->copy_stream),
                               reinterpret_cast<CUdeviceptr>(L->d_slot_ready + s), gen, 0);
        if (r == CUDA_SUCCESS) return WISP_OK;
    }
    // fallback: a 4-byte copy from a pinned ring, ordered after the weights
    uint32_t *src = L->h_flag_ring + (L->flag_idx.fetch_add(1) % kFlagRing);
    *src = gen;
    WISP_CUDA_TRY(cudaMemcpyAsync(L->d_slot_ready + s, src, sizeof(uint32_t), cudaMemcpyHostToDevice,
                                  L->copy_stream));
    return WISP_OK;
}

// ---------------------------------------------------------------------------
// Page-in engine: one host thread per device serving every layer's async
// forwards.  A task is one forward; tasks of one layer are served in order,
// tasks of different layers independently.
// ---------------------------------------------------------------------------
struct PageTask {
    wisp_layer *L;
    uint32_t seq;
    int T;
    int slot;  // mailbox of this forward
    bool loaded = false;
    int nmiss = 0, next = 0;
    std::vector<int32_t> recs;
    std::chrono::steady_clock::time_point last;
};

class Engine {
  public:
    explicit Engine(int dev) : dev_(dev) {
        th_ = std::thread([this] { run(); });
        th_.detach();
    }

    void submit(wisp_layer *L, uint32_t seq, int T, int slot) {
        auto t = std::make_unique<PageTask>();
        t->L = L;
        t->seq = seq;
        t->T = T;
        t->slot = slot;
        t->last = std::chrono::steady_clock::now();
        L->pending.fetch_add(1);
        {
            std::lock_guard<std::mutex> lk(mu_);
            q_.push_back(std::move(t));
        }
        cv_.notify_one();
    }

    // Wait until no task of L is queued (bounded).
    bool wait_idle(wisp_layer *L, long long limit_ns) {
        auto t0 = std::chrono::steady_clock::now();
        while (L->pending.load() > 0) {
            if (std::chrono::duration_cast<std::chrono::nanoseconds>(std::chrono::steady_clock::now() - t0)
                    .count() > limit_ns)
                return false;
            std::this_thread::yield();
        }
        return true;
    }

  private:
    // 0: nothing to do yet, 1: progressed, 2: finished
    int step(PageTask &t) {
        wisp_layer *L = t.L;
        volatile int32_t *mb = L->h_mb + (long)t.slot * L->mb_words;
        const auto now = std::chrono::steady_clock::now();
        const long long host_limit = L->wait_ns + 5LL * 1000 * 1000 * 1000;
        auto timed_out = [&] {
            return std::chrono::duration_cast<std::chrono::nanoseconds>(now - t.last).count() > host_limit;
        };
        auto give_up = [&](int code) {
            int z = 0;
            L->host_status.compare_exchange_strong(z, code);
            return 2;
        };
        if (*reinterpret_cast<volatile int32_t *>(L->h_status) != 0) return 2;  // the kernel gave up
        if (!t.loaded) {
            if ((uint32_t)mb[7] != t.seq) return timed_out() ? give_up(WISP_ERR_TIMEOUT) : 0;
            std::atomic_thread_fence(std::memory_order_acquire);
            const int status = mb[0];
            const int nmiss = mb[2];
            if (status != WISP_OK || nmiss == 0) return 2;
            const long off = mailbox_miss_offset(t.T);
            t.recs.resize((size_t)nmiss * kMbRec);
            for (size_t i = 0; i < t.recs.size(); ++i) t.recs[i] = mb[off + (long)i];
            t.nmiss = nmiss;
            t.loaded = true;
            t.last = now;
        }
        int progressed = 0;
        while (t.next < t.nmiss) {
            const int32_t *rec = t.recs.data() + (size_t)kMbRec * t.next;
            const int wg = rec[3];
            if (wg >= 0) {
                const unsigned long long need = ((unsigned long long)t.seq << 32) | (unsigned)(wg + 1);
                const unsigned long long have = *reinterpret_cast<volatile unsigned long long *>(L->h_done);
                if (have < need) return timed_out() ? give_up(WISP_ERR_TIMEOUT) : progressed;
            }
            if (L->drop_pageins.load() > 0) {
                L->drop_pageins.fetch_sub(1);  // test fault: this slot's flag is never raised
            } else if (issue_pagein(L, rec[0], rec[1], (uint32_t)rec[4]) != WISP_OK) {
                return give_up(WISP_ERR_CUDA);
            }
            ++t.next;
            t.last = now;
            progressed = 1;
        }
        return 2;
    }

    void run() {
        cudaSetDevice(dev_);
        std::call_once(g_write32_once, init_write32);
        std::vector<PageTask *> snap, done;
        std::vector<wisp_layer *> seen;
        for (;;) {
            {
                std::unique_lock<std::mutex> lk(mu_);
                cv_.wait(lk, [&] { return !q_.empty(); });
                snap.clear();
                for (auto &p : q_) snap.push_back(p.get());
            }
            bool progress = false;
            seen.clear();
            done.clear();
            for (PageTask *t : snap) {
                if (std::find(seen.begin(), seen.end(), t->L) != seen.end()) continue;
                seen.push_back(t->L);
                const int r = step(*t);
                if (r) progress = true;
                if (r == 2) done.push_back(t);
            }
            if (!done.empty()) {
                std::lock_guard<std::mutex> lk(mu_);
                for (PageTask *t : done) {
                    wisp_layer *L = t->L;
                    L->mb_busy[t->slot].store(0);
                    auto it = std::find_if(q_.begin(), q_.end(), [&](const std::unique_ptr<PageTask> &p) {
                        return p.get() == t;
                    });
                    q_.erase(it);
                    L->pending.fetch_sub(1);
                }
            }
            if (!progress) std::this_thread::yield();
        }
    }

    int dev_;
    std::mutex mu_;
    std::condition_variable cv_;
    std::deque<std::unique_ptr<PageTask>> q_;
    std::thread th_;
};

Engine *engine_for(int dev) {
    static std::mutex mu;
    static Engine *engines[64] = {};
    std::lock_guard<std::mutex> lk(mu);
    if (!engines[dev]) engines[dev] = new Engine(dev);  // lives until process exit
    return engines[dev];
}

// ---------------------------------------------------------------------------
// allocation helpers
// ---------------------------------------------------------------------------
void free_ws(wisp_layer *L) {
    for (void *p : {(void *)L->d_slots, (void *)L->d_grp_start, (void *)L->d_grp_nu,
                    (void *)L->d_grp_nhit, (void *)L->d_u_slot,
                    (void *)L->d_u_gen, (void *)L->d_u_off, (void *)L->d_u_pairs, (void *)L->d_counters,
                    (void *)L->d_dev_hdr, (void *)L->d_act, (void *)L->d_y, (void *)L->d_xperm,
                    (void *)L->d_actperm, (void *)L->d_ready, (void *)L->d_combined, (void *)L->d_route,
                    (void *)L->d_xq,
                    (void *)L->d_aq, (void *)L->d_xs, (void *)L->d_as})
        cudaFree(p);
    L->d_xq = L->d_aq = nullptr;
    L->d_xs = L->d_as = nullptr;
    if (L->h_mb) cudaFreeHost(L->h_mb);
    L->d_slots = L->d_grp_start = L->d_grp_nu = L->d_grp_nhit = L->d_u_slot = L->d_u_gen = L->d_u_off =
        L->d_u_pairs = L->d_counters = L->d_dev_hdr = nullptr;
    L->d_act = L->d_y = L->d_xperm = L->d_actperm = nullptr;
    L->d_ready = L->d_combined = nullptr;
    L->d_route = nullptr;
    L->h_mb = L->d_mb = nullptr;
    L->wsT = -1;
    L->wsK = 0;
}

// Grow the per-call workspace (geometrically, so a varying batch settles).
// Frees and allocations wait for the whole device first: cudaFree and
// cudaFreeHost synchronise implicitly and stall the page-in thread's copy
// calls meanwhile, so one issued while another layer's forward kernel waits
// for its page-ins would hold that kernel until its wait limit runs out.
// cudaDeviceSynchronize waits without stalling the page-in thread.
int ensure_ws(wisp_layer *L, int T, int K) {
    if (T <= L->wsT && K <= L->wsK) return WISP_OK;
    const int nT = std::max({T, L->wsT > 0 ? 2 * L->wsT : 0, 16});
    const int nK = std::max({K, L->wsK, 8});
    WISP_CUDA_TRY(cudaDeviceSynchronize());
    free_ws(L);
    const size_t P = std::max<size_t>((size_t)nT * nK, 1);
    WISP_CUDA_TRY(cudaMalloc(&L->d_slots, sizeof(int32_t) * P));
    WISP_CUDA_TRY(cudaMalloc(&L->d_grp_start, sizeof(int32_t) * (nT + 1)));
    WISP_CUDA_TRY(cudaMalloc(&L->d_grp_nu, sizeof(int32_t) * (nT + 1)));
    WISP_CUDA_TRY(cudaMalloc(&L->d_grp_nhit, sizeof(int32_t) * (nT + 1)));
    WISP_CUDA_TRY(cudaMalloc(&L->d_u_slot, sizeof(int32_t) * P));
    WISP_CUDA_TRY(cudaMalloc(&L->d_u_gen, sizeof(int32_t) * P));
    WISP_CUDA_TRY(cudaMalloc(&L->d_u_off, sizeof(int32_t) * (P + nT + 1)));
    WISP_CUDA_TRY(cudaMalloc(&L->d_u_pairs, sizeof(int32_t) * P));
    WISP_CUDA_TRY(cudaMalloc(&L->d_dev_hdr, sizeof(int32_t) * kHdrWords));
    const int H = std::max(L->H, 8), I = std::max(L->I, 8);
    const int nblk = (H + 3) / 4;  // row quads (forward kernel) >= row octets (decode kernels)
    WISP_CUDA_TRY(cudaMalloc(&L->d_counters, sizeof(int32_t) * nblk));
    WISP_CUDA_TRY(cudaMemset(L->d_counters, 0, sizeof(int32_t) * nblk));
    if (L->fp8) {
        WISP_CUDA_TRY(cudaMalloc(&L->d_xq, (size_t)nT * H));
        WISP_CUDA_TRY(cudaMalloc(&L->d_xs, sizeof(float) * (size_t)nT * (H / kFp8Block)));
        WISP_CUDA_TRY(cudaMalloc(&L->d_aq, P * (size_t)I));
        WISP_CUDA_TRY(cudaMalloc(&L->d_as, sizeof(float) * P * (I / kFp8Block)));
    }
    if (L->H > 0 && L->I > 0) {
        // two halves, by launch parity (the one-launch forward polls its half)
        WISP_CUDA_TRY(cudaMalloc(&L->d_act, sizeof(__nv_bfloat16) * 2 * P * I));
        L->act_dirty = true;
        WISP_CUDA_TRY(cudaMalloc(&L->d_y, sizeof(__nv_bfloat16) * P * H));
        if (prefill_shapes_supported(L->H, L->I)) {
            WISP_CUDA_TRY(cudaMalloc(&L->d_xperm, sizeof(__nv_bfloat16) * P * H));
            WISP_CUDA_TRY(cudaMalloc(&L->d_actperm, sizeof(__nv_bfloat16) * P * I));
            WISP_CUDA_TRY(cudaMalloc(&L->d_ready, sizeof(uint32_t) * 2 * kBatchReadyWords));
            WISP_CUDA_TRY(cudaMemset(L->d_ready, 0, sizeof(uint32_t) * 2 * kBatchReadyWords));
            WISP_CUDA_TRY(cudaMalloc(&L->d_combined, sizeof(uint32_t) * 2 * batch_done_words(L->H)));
            WISP_CUDA_TRY(cudaMemset(L->d_combined, 0, sizeof(uint32_t) * 2 * batch_done_words(L->H)));
            L->ready_parity = 0;
            const size_t rw = 2 * (2 * (size_t)L->E + 1) + 2;
            WISP_CUDA_TRY(cudaMalloc(&L->d_route, sizeof(int32_t) * rw));
            WISP_CUDA_TRY(cudaMemset(L->d_route, 0, sizeof(int32_t) * rw));
            L->route_parity = 0;
        }
    }
    const long words = (mailbox_words(nT, nK) + 31) & ~31L;
    WISP_CUDA_TRY(cudaHostAlloc(&L->h_mb, sizeof(int32_t) * words * kMbRing, cudaHostAllocMapped));
    std::fill(L->h_mb, L->h_mb + words * kMbRing, 0);
    L->mb_words = words;
    WISP_CUDA_TRY(cudaHostGetDevicePointer((void **)&L->d_mb, L->h_mb, 0));
    L->wsT = nT;
    L->wsK = nK;
    return WISP_OK;
}

int ensure_events(wisp_layer *L, int G) {
    while ((int)L->ev_group.size() < G) {
        cudaEvent_t a, b;
        WISP_CUDA_TRY(cudaEventCreateWithFlags(&a, cudaEventDisableTiming));
        WISP_CUDA_TRY(cudaEventCreateWithFlags(&b, cudaEventDisableTiming));
        L->ev_group.push_back(a);
        L->ev_copy.push_back(b);
    }
    return WISP_OK;
}

int alloc_slots(wisp_layer *L, int cap) {
    WISP_CUDA_TRY(cudaMalloc(&L->d13, (size_t)cap * L->b13));
    WISP_CUDA_TRY(cudaMalloc(&L->d2, (size_t)cap * L->b2));
    if (L->fp8) {
        WISP_CUDA_TRY(cudaMalloc(&L->ds13, (size_t)cap * L->bs13));
        WISP_CUDA_TRY(cudaMalloc(&L->ds2, (size_t)cap * L->bs2));
    }
    WISP_CUDA_TRY(cudaMalloc(&L->d_s2e, sizeof(int32_t) * cap));
    WISP_CUDA_TRY(cudaMalloc(&L->d_tick, sizeof(int64_t) * cap));
    WISP_CUDA_TRY(cudaMalloc(&L->d_slot_gen, sizeof(uint32_t) * cap));
    WISP_CUDA_TRY(cudaMalloc(&L->d_slot_ready, sizeof(uint32_t) * cap));
    WISP_CUDA_TRY(cudaMemset(L->d_s2e, 0xff, sizeof(int32_t) * cap));
    WISP_CUDA_TRY(cudaMemset(L->d_tick, 0, sizeof(int64_t) * cap));
    WISP_CUDA_TRY(cudaMemset(L->d_slot_gen, 0, sizeof(uint32_t) * cap));
    WISP_CUDA_TRY(cudaMemset(L->d_slot_ready, 0, sizeof(uint32_t) * cap));
    return WISP_OK;
}

void fill_pager_params(wisp_layer *L, PagerParams &p, const void *ids, int ids64, int T, int K,
                       int single_group, int count_forward) {
    p = PagerParams{};
    p.ids = ids;
    p.ids64 = ids64;
    p.T = T;
    p.K = K;
    p.E = L->E;
    p.cap = L->cap;
    p.mode = L->mode;
    p.count_forward = count_forward;
    p.single_group = single_group;
    if (++L->seq == 0) ++L->seq;  // 0 marks a mailbox being rewritten
    p.seq = L->seq;
    p.s2e = L->d_s2e;
    p.tick = L->d_tick;
    p.emap = L->d_emap;
    p.hdr = L->d_hdr;
    p.slot_gen = L->d_slot_gen;
    p.last_unique = L->d_last_unique;
    p.slots = L->d_slots;
    p.grp_start = L->d_grp_start;
    p.grp_nu = L->d_grp_nu;
    p.grp_nhit = L->d_grp_nhit;
    p.u_slot = L->d_u_slot;
    p.u_gen = L->d_u_gen;
    p.u_off = L->d_u_off;
    p.u_pairs = L->d_u_pairs;
    p.dev_hdr = L->d_dev_hdr;
    p.mb = L->d_mb;
}

// Wait for every async forward of L (kernels and page-ins).
int drain(wisp_layer *L) {
    WISP_CUDA_TRY(cudaEventSynchronize(L->ev_last));
    if (!engine_for(L->dev)->wait_idle(L, L->wait_ns + 10LL * 1000 * 1000 * 1000))
        return fail(WISP_ERR_TIMEOUT, "wisp: page-in engine did not drain");
    WISP_CUDA_TRY(cudaStreamSynchronize(L->copy_stream));
    return WISP_OK;
}

// Restart the pager cold after a failed forward: no slot resident, the
// grid-barrier words and slot flags consistent again; clock and counters kept.
int reset_cold(wisp_layer *L) {
    WISP_CUDA_TRY(cudaDeviceSynchronize());
    WISP_CUDA_TRY(cudaMemset(L->d_bar, 0, sizeof(unsigned int) * kBarWords));
    WISP_CUDA_TRY(cudaMemset(L->d_flow, 0, sizeof(unsigned int) * kFlowWords));
    if (L->mode != WISP_MODE_RESIDENT) {
        // a resident layer keeps its identity map: its slots still hold every
        // expert (only wisp_prime_identity writes them)
        WISP_CUDA_TRY(cudaMemset(L->d_s2e, 0xff, sizeof(int32_t) * L->cap));
        WISP_CUDA_TRY(cudaMemset(L->d_emap, 0xff, sizeof(int32_t) * L->E));
        WISP_CUDA_TRY(cudaMemset(L->d_tick, 0, sizeof(int64_t) * L->cap));
    }
    WISP_CUDA_TRY(cudaMemcpy(L->d_slot_ready, L->d_slot_gen, sizeof(uint32_t) * L->cap,
                             cudaMemcpyDeviceToDevice));
    const int nblk = (std::max(L->H, 8) + 3) / 4;
    WISP_CUDA_TRY(cudaMemset(L->d_counters, 0, sizeof(int32_t) * nblk));
    WISP_CUDA_TRY(cudaDeviceSynchronize());
    L->act_dirty = true;
    return WISP_OK;
}

// Errors of earlier async forwards (device sticky status, page-in engine).
int take_errors(wisp_layer *L) {
    volatile int32_t *stw = L->h_status;
    const int dev_st = *stw;
    const int host_st = L->host_status.exchange(0);
    if (!dev_st && !host_st) return WISP_OK;
    const int code = dev_st ? dev_st : host_st;
    const int rc = drain(L);
    *stw = 0;
    if (code == WISP_ERR_BAD_EXPERT) {
        // the pager rejected the ids before touching any state
        if (!rc) {
            cudaMemset(L->d_bar, 0, sizeof(unsigned int) * kBarWords);
            cudaMemset(L->d_flow, 0, sizeof(unsigned int) * kFlowWords);
            cudaDeviceSynchronize();
        }
        L->act_dirty = true;
        return fail(code, "wisp: an earlier forward routed an expert id outside [0, " +
                              std::to_string(L->E) + ")");
    }
    reset_cold(L);
    return fail(code, code == WISP_ERR_TIMEOUT
                          ? "wisp: an earlier forward gave up waiting (page-in or grid barrier ran past "
                            "the wait limit); the layer restarted with no expert resident"
                          : "wisp: an earlier forward's page-in failed; the layer restarted with no "
                            "expert resident");
}

// Run K1 alone and wait for it; returns the pager status (synchronous path).
int run_pager(wisp_layer *L, const void *ids, int ids64, int T, int K, int single_group,
              int count_forward, cudaStream_t stream) {
    int rc = drain(L);
    if (rc) return rc;
    rc = ensure_ws(L, T, K);
    if (rc) return rc;
    PagerParams p;
    fill_pager_params(L, p, ids, ids64, T, K, single_group, count_forward);
    WISP_CUDA_TRY(cudaStreamWaitEvent(stream, L->ev_copies, 0));
    rc = launch_pager(p, stream);
    if (rc) return rc;
    ++L->launches;
    WISP_CUDA_TRY(cudaEventRecord(L->ev_pager, stream));
    L->last_stream_set = false;
    WISP_CUDA_TRY(cudaEventSynchronize(L->ev_pager));
    const int status = ((volatile int32_t *)L->h_mb)[0];
    if (status == WISP_OK && count_forward && L->mode != WISP_MODE_RESIDENT) {
        for (int w = 0; w < 32; ++w) L->h_last_unique[w] = (uint32_t)((volatile int32_t *)L->h_mb)[kMbUnique + w];
        L->last_unique_host = true;
    }
    if (status == WISP_ERR_OVERFLOW)
        return fail(WISP_ERR_OVERFLOW,
                    "wisp: per-kernel-call working set exceeds cap_experts (" +
                        std::to_string(L->cap) +
                        "); a single call routes to more unique experts than the cap, so the "
                        "forward cannot sub-batch it");
    if (status == WISP_ERR_BAD_EXPERT)
        return fail(WISP_ERR_BAD_EXPERT,
                    "wisp: routed expert id outside [0, " + std::to_string(L->E) + ")");
    if (status != WISP_OK) return fail(WISP_ERR_CUDA, "wisp: pager did not complete");
    return WISP_OK;
}

// Which kernels run a call's expert compute.  The choice depends on the
// call's size (T * k) only, not on its grouping, so outputs stay
// byte-identical across caps, modes and slot placements.
enum class Path { kDecode, kBatchTC, kPrefillTC, kFp8 };
Path compute_path(const wisp_layer *L, int T, int K) {
    const long pairs = (long)T * K;
    if (L->fp8) return Path::kFp8;
    if (!prefill_shapes_supported(L->H, L->I) || L->compute_class == 1) return Path::kDecode;
    if (pairs >= kPrefillMinPairs) return Path::kPrefillTC;
    if (L->compute_class == 2) return Path::kBatchTC;
    if (pairs >= L->tc_min_pairs) return Path::kBatchTC;
    return Path::kDecode;
}

// A group of the call for the tensor-core launchers.
PrefillGroup tc_group(const wisp_layer *L, const void *x, const float *w, void *out, int g, int t0, int t1,
                      int K, int nu_bound, const int32_t *pager_status) {
    const int64_t p0 = (int64_t)t0 * K;
    PrefillGroup pg{};
    pg.x = reinterpret_cast<const __nv_bfloat16 *>(x);
    pg.w13 = reinterpret_cast<const __nv_bfloat16 *>(L->d13);
    pg.w2 = reinterpret_cast<const __nv_bfloat16 *>(L->d2);
    pg.slots = L->cap;
    pg.u_off = L->d_u_off + p0 + g;
    pg.u_pairs = L->d_u_pairs + p0;
    pg.u_slot = L->d_u_slot + p0;
    pg.nu_dev = L->d_grp_nu + g;
    pg.pager_status = pager_status;
    pg.u_gen = nullptr;
    pg.slot_ready = L->d_slot_ready;
    pg.nu = nu_bound;
    pg.npairs = (t1 - t0) * K;
    pg.t0 = t0;
    pg.t1 = t1;
    pg.K = K;
    pg.H = L->H;
    pg.I = L->I;
    pg.topk_w = w;
    pg.x_perm = L->d_xperm;
    pg.act_perm = L->d_actperm;
    pg.perm_rows = L->wsT * L->wsK;
    pg.y = L->d_y;
    pg.out = reinterpret_cast<__nv_bfloat16 *>(out);
    pg.status = L->d_status;
    pg.wait_ns = L->wait_ns;
    pg.trace = L->trace;
    return pg;
}

// The counter halves of the next weight-stationary launch (it zeroes the
// other halves for the launch after it); flips the parity, which the caller
// flips back when the launch is not queued (those halves were not zeroed).
BatchCounters take_counters(wisp_layer *L) {
    BatchCounters c{};
    if (!L->d_ready || !L->d_combined) return c;
    const size_t nd = (size_t)batch_done_words(L->H);
    const int cur = L->ready_parity, nxt = cur ^ 1;
    c.ready = L->d_ready + (size_t)cur * kBatchReadyWords;
    c.ready_next = L->d_ready + (size_t)nxt * kBatchReadyWords;
    c.done = L->d_combined + (size_t)cur * nd;
    c.done_next = L->d_combined + (size_t)nxt * nd;
    L->ready_parity = nxt;
    return c;
}

int launch_tc_group(wisp_layer *L, Path path, const PrefillGroup &pg, cudaStream_t stream) {
    if (path == Path::kBatchTC) {
        const int rc = launch_batch_group(pg, take_counters(L), stream);
        if (!rc)
            L->launches += kBatchKernelsPerGroup;
        else
            L->ready_parity ^= 1;  // not queued: the next launch takes these halves again
        return rc;
    }
    const int rc = launch_prefill_group(pg, stream);
    if (!rc) L->launches += kPrefillKernelsPerGroup;
    return rc;
}

// Synchronous path after run_pager: page-ins per group (write-after-read via
// group events) and, when `compute` is set, the per-group decode kernels.
int page_and_compute(wisp_layer *L, const void *x, const float *w, int T, int K, void *out,
                     cudaStream_t stream, bool compute) {
    const int32_t *mb = L->h_mb;
    const int G = mb[1], nmiss = mb[2];
    const int32_t *grp = mb + kMbHeader;
    const int32_t *nu = grp + (T + 1);
    const int32_t *rec = mb + mailbox_miss_offset(T);
    int rc = ensure_events(L, std::max(G, 1));
    if (rc) return rc;
    const Path path = compute_path(L, T, K);
    if (compute && path == Path::kFp8 && T > 0) {
        // the call's tokens, quantised once for every group
        rc = launch_fp8_quant_rows(reinterpret_cast<const __nv_bfloat16 *>(x), T, L->H, L->d_xq, L->d_xs, stream);
        if (rc) return rc;
        ++L->launches;
    }
    int mi = 0;
    for (int g = 0; g < G; ++g) {
        const int t0 = grp[g], t1 = grp[g + 1];
        int wait_g = -1, m0 = mi;
        while (mi < nmiss && rec[kMbRec * mi + 2] == g) {
            wait_g = std::max(wait_g, (int)rec[kMbRec * mi + 3]);
            ++mi;
        }
        // the weight-stationary kernel waits inside for each expert's slot (its
        // resident experts compute while the misses stream in); every other
        // kernel waits for the group's copies on the stream
        const bool slot_waits = compute && path == Path::kBatchTC && t1 > t0 && nu[g] > 0;
        if (mi > m0) {
            if (wait_g >= 0) WISP_CUDA_TRY(cudaStreamWaitEvent(L->copy_stream, L->ev_group[wait_g], 0));
            for (int m = m0; m < mi; ++m) {
                rc = issue_pagein(L, rec[kMbRec * m], rec[kMbRec * m + 1], (uint32_t)rec[kMbRec * m + 4]);
                if (rc) return rc;
            }
            WISP_CUDA_TRY(cudaEventRecord(L->ev_copy[g], L->copy_stream));
            if (!slot_waits) WISP_CUDA_TRY(cudaStreamWaitEvent(stream, L->ev_copy[g], 0));
        }
        const bool tensor_cores = path == Path::kBatchTC || path == Path::kPrefillTC;
        if (compute && t1 > t0 && nu[g] > 0 && tensor_cores) {
            // tensor-core kernels (gather, gate-up + SiLU-mul, down, combine)
            PrefillGroup pg = tc_group(L, x, w, out, g, t0, t1, K, nu[g], nullptr);
            if (slot_waits && mi > m0) pg.u_gen = L->d_u_gen + (int64_t)t0 * K;
            rc = launch_tc_group(L, path, pg, stream);
            if (rc) return rc;
        } else if (compute && t1 > t0 && nu[g] > 0 && path == Path::kFp8) {
            const int64_t p0 = (int64_t)t0 * K;
            Fp8Group fg{};
            fg.xq = L->d_xq;
            fg.xs = L->d_xs;
            fg.w13 = reinterpret_cast<const uint8_t *>(L->d13);
            fg.s13 = reinterpret_cast<const float *>(L->ds13);
            fg.w2 = reinterpret_cast<const uint8_t *>(L->d2);
            fg.s2 = reinterpret_cast<const float *>(L->ds2);
            fg.u_slot = L->d_u_slot + p0;
            fg.u_off = L->d_u_off + p0 + g;
            fg.u_pairs = L->d_u_pairs + p0;
            fg.nu = L->d_grp_nu + g;
            fg.topk_w = w;
            fg.act = L->d_act;
            fg.aq = L->d_aq;
            fg.as = L->d_as;
            fg.y = L->d_y;
            fg.out = reinterpret_cast<__nv_bfloat16 *>(out);
            fg.counters = L->d_counters;
            fg.K = K;
            fg.H = L->H;
            fg.I = L->I;
            fg.t0 = t0;
            fg.t1 = t1;
            rc = launch_fp8_group(fg, nu[g], stream);
            if (rc) return rc;
            L->launches += kFp8KernelsPerGroup;
            L->act_dirty = true;
        } else if (compute && t1 > t0 && nu[g] > 0) {
            const int64_t p0 = (int64_t)t0 * K;
            GroupCompute gc{};
            gc.x = reinterpret_cast<const __nv_bfloat16 *>(x);
            gc.w13 = reinterpret_cast<const __nv_bfloat16 *>(L->d13);
            gc.w2 = reinterpret_cast<const __nv_bfloat16 *>(L->d2);
            gc.u_slot = L->d_u_slot + p0;
            gc.u_off = L->d_u_off + p0 + g;
            gc.u_pairs = L->d_u_pairs + p0;
            gc.nu = L->d_grp_nu + g;
            gc.topk_w = w;
            gc.act = L->d_act;
            gc.y = L->d_y;
            gc.out = reinterpret_cast<__nv_bfloat16 *>(out);
            gc.counters = L->d_counters;
            gc.K = K;
            gc.H = L->H;
            gc.I = L->I;
            gc.t0 = t0;
            gc.t1 = t1;
            rc = launch_decode_group(gc, nu[g], stream);
            if (rc) return rc;
            L->launches += kDecodeKernelsPerGroup;
            L->act_dirty = true;
        }
        WISP_CUDA_TRY(cudaEventRecord(L->ev_group[g], stream));
    }
    WISP_CUDA_TRY(cudaEventRecord(L->ev_copies, L->copy_stream));
    ++L->copy_gen;
    WISP_CUDA_TRY(cudaEventRecord(L->ev_last, stream));
    L->last_stream_set = false;  // the next resident forward waits for this work explicitly
    return WISP_OK;
}

// Resident layers run the tensor-core paths without a host round trip.  Up
// to 512 pairs the weight-stationary kernel routes the call itself (no pager
// launch: a resident layer's pager step only counts the forward, which that
// kernel does).  Larger calls: the pager (one group, slots fixed) leaves the
// expert lists and count on the device and the GEMM kernels read them there.
// A rejected call is skipped and its status lands in the sticky word,
// reported by the next call or synchronize.
// Order `stream` after the layer's previous forward and its copies (the
// workspace and the slots), unless stream order already does; then note the
// stream as the layer's last.
int order_resident(wisp_layer *L, cudaStream_t stream) {
    if (!(L->last_stream_set && L->last_stream == stream && L->copy_waited == L->copy_gen)) {
        WISP_CUDA_TRY(cudaStreamWaitEvent(stream, L->ev_last, 0));
        WISP_CUDA_TRY(cudaStreamWaitEvent(stream, L->ev_copies, 0));
        L->copy_waited = L->copy_gen;
    }
    L->last_stream = stream;
    L->last_stream_set = true;
    return WISP_OK;
}

int forward_tc_resident(wisp_layer *L, Path path, const void *x, const float *w, const void *ids, int ids64,
                        int T, int K, void *out, cudaStream_t stream) {
    if (T > L->wsT || K > L->wsK) {
        int rc = drain(L);
        if (rc) return rc;
        rc = ensure_ws(L, T, K);
        if (rc) return rc;
    }
    // the layer's workspace: after its previous forward, whichever stream that used
    int orc = order_resident(L, stream);
    if (orc) return orc;
    if (path == Path::kBatchTC) {
        BatchRoute r{};
        r.ids = ids;
        r.ids64 = ids64;
        r.E = L->E;
        r.count_forward = 1;
        r.emap = L->d_emap;
        r.hdr = L->d_hdr;
        r.dev_status = L->d_dev_hdr + kHdrStatus;
        const int nu_bound = (int)std::min<long>(L->E, (long)T * K);
        const PrefillGroup pg = tc_group(L, x, w, out, 0, 0, T, K, nu_bound, nullptr);
        int rc = launch_batch_resident(pg, r, take_counters(L), stream);
        if (rc) {
            L->ready_parity ^= 1;  // not queued: the next launch takes these halves again
            return rc;
        }
        L->launches += kBatchKernelsResident;
        WISP_CUDA_TRY(cudaEventRecord(L->ev_last, stream));
        return WISP_OK;
    }
    // token-major GEMMs: a routing kernel writes the group lists, as the pager
    // would for an all-resident call, and counts the forward (no LRU state: a
    // resident layer pages nothing)
    BatchRoute r{};
    r.ids = ids;
    r.ids64 = ids64;
    r.E = L->E;
    r.count_forward = 1;
    r.emap = L->d_emap;
    r.hdr = L->d_hdr;
    r.dev_status = L->d_dev_hdr + kHdrStatus;
    const size_t half = 2 * (size_t)L->E + 1;
    PrefillLists lists{L->d_u_off, L->d_u_pairs, L->d_u_slot, L->d_grp_nu,
                       L->d_route + L->route_parity * half, L->d_route + (L->route_parity ^ 1) * half,
                       reinterpret_cast<uint32_t *>(L->d_route + 2 * half)};
    const int nu_bound = (int)std::min<long>(L->E, (long)T * K);
    const int rc = launch_prefill_resident(tc_group(L, x, w, out, 0, 0, T, K, nu_bound, L->d_dev_hdr + kHdrStatus),
                                           r, lists, stream);
    if (rc) return rc;
    L->route_parity ^= 1;
    L->launches += kPrefillKernelsResident;
    WISP_CUDA_TRY(cudaEventRecord(L->ev_last, stream));
    return WISP_OK;
}

int forward_async(wisp_layer *L, const void *x, const float *w, const void *ids, int ids64, int T,
                  int K, void *out, cudaStream_t stream) {
    if (T > L->wsT || K > L->wsK) {
        int rc = drain(L);
        if (rc) return rc;
        rc = ensure_ws(L, T, K);
        if (rc) return rc;
    }
    ForwardParams fp{};
    fill_pager_params(L, fp.pg, ids, ids64, T, K, 0, 1);
    fp.gc.x = reinterpret_cast<const __nv_bfloat16 *>(x);
    fp.gc.w13 = reinterpret_cast<const __nv_bfloat16 *>(L->d13);
    fp.gc.w2 = reinterpret_cast<const __nv_bfloat16 *>(L->d2);
    fp.gc.topk_w = w;
    // activation half of this launch's parity; the launch resets the other
    // half to kActEmpty for the next one
    const size_t act_half = (size_t)L->wsT * L->wsK * (size_t)std::max(L->I, 0);
    if (L->act_dirty && act_half) {
        WISP_CUDA_TRY(cudaMemsetAsync(L->d_act, 0xff, sizeof(__nv_bfloat16) * 2 * act_half, stream));
        L->act_dirty = false;
    }
    fp.gc.act = L->d_act + (size_t)L->kparity * act_half;
    fp.act_reset = reinterpret_cast<uint32_t *>(L->d_act + (size_t)(L->kparity ^ 1) * act_half);
    fp.act_reset_words = (long)(act_half / 2);
    fp.gc.y = L->d_y;
    fp.gc.out = reinterpret_cast<__nv_bfloat16 *>(out);
    fp.gc.counters = L->d_counters;
    fp.gc.K = K;
    fp.gc.H = L->H;
    fp.gc.I = L->I;
    fp.slot_ready = L->d_slot_ready;
    fp.bar = L->d_bar;
    fp.done_word = L->d_done;
    fp.wait_ns = L->wait_ns;
    fp.status_word = L->d_status;
    fp.trace = L->trace;
    fp.flow = L->d_flow;
    fp.epoch = L->kparity;
    const bool paged = L->mode == WISP_MODE_PAGED;
    fp.publish = paged ? 1 : 0;
    int slot = 0;
    if (paged) {
        // a mailbox no page-in task still reads (the engine frees them in order)
        slot = L->mb_next;
        L->mb_next = (slot + 1) % kMbRing;
        const auto t0 = std::chrono::steady_clock::now();
        while (L->mb_busy[slot].load()) {
            if (std::chrono::duration_cast<std::chrono::nanoseconds>(std::chrono::steady_clock::now() - t0)
                    .count() > L->wait_ns + 5LL * 1000 * 1000 * 1000)
                return fail(WISP_ERR_TIMEOUT, "wisp: page-in engine stalled (mailbox still in use)");
            std::this_thread::yield();
        }
        L->mb_busy[slot].store(1);
    }
    fp.pg.mb = L->d_mb + (long)slot * L->mb_words;
    if (paged) L->last_unique_host = false;  // this forward's set is known on the device only
    if (paged) {
        WISP_CUDA_TRY(cudaStreamWaitEvent(stream, L->ev_last, 0));  // the workspace, whichever stream used it last
        WISP_CUDA_TRY(cudaStreamWaitEvent(stream, L->ev_copies, 0));
        L->last_stream_set = false;
    } else {
        const int orc = order_resident(L, stream);
        if (orc) return orc;
    }
    int rc = launch_forward(fp, T, stream);
    if (rc) {
        if (paged) L->mb_busy[slot].store(0);
        return rc;
    }
    L->kparity ^= 1;
    ++L->launches;
    WISP_CUDA_TRY(cudaEventRecord(L->ev_last, stream));
    if (paged) engine_for(L->dev)->submit(L, fp.pg.seq, T, slot);
    return WISP_OK;
}

}  // namespace

static int layer_create_impl(int32_t num_experts, int32_t cap_experts, int32_t hidden, int32_t inter,
                             int64_t w13_expert_bytes, int64_t w2_expert_bytes, const void *host_w13,
                             const void *host_w2, int32_t device, int32_t mode, wisp_layer **out,
                             const void *host_s13 = nullptr, const void *host_s2 = nullptr) {
    const bool fp8 = host_s13 != nullptr;
    if (!out) return fail(WISP_ERR_INVALID, "wisp_layer_create: out is NULL");
    *out = nullptr;
    if (num_experts < 1 || num_experts > 1024)
        return fail(WISP_ERR_INVALID, "wisp_layer_create: num_experts must be in [1, 1024]");
    if (cap_experts < 1 || cap_experts > num_experts)
        return fail(WISP_ERR_INVALID, "wisp_layer_create: cap_experts must be in [1, num_experts]");
    if (mode != WISP_MODE_PAGED && mode != WISP_MODE_RESIDENT)
        return fail(WISP_ERR_INVALID, "wisp_layer_create: unknown mode");
    if (mode == WISP_MODE_RESIDENT && cap_experts != num_experts)
        return fail(WISP_ERR_INVALID, "wisp_layer_create: resident mode needs cap == num_experts");
    if (w13_expert_bytes <= 0 || w2_expert_bytes <= 0 || !host_w13 || !host_w2)
        return fail(WISP_ERR_INVALID, "wisp_layer_create: empty expert weights");
    if (hidden < 0 || inter < 0) return fail(WISP_ERR_INVALID, "wisp_layer_create: negative shape");
    if (hidden > 0 && inter > 0 && !fp8) {
        if (hidden % 8 || inter % 8)
            return fail(WISP_ERR_UNSUPPORTED, "wisp_layer_create: hidden and inter must be multiples of 8");
        if (w13_expert_bytes != 2LL * 2 * inter * hidden || w2_expert_bytes != 2LL * hidden * inter)
            return fail(WISP_ERR_INVALID,
                        "wisp_layer_create: expert bytes do not match bf16 [2I,H] / [H,I]");
    }
    if (device < 0 || device >= 64) return fail(WISP_ERR_INVALID, "wisp_layer_create: bad device");
    DeviceGuard guard(device);
    std::call_once(g_write32_once, init_write32);
    // other layers' forwards may be in flight: let them finish before the
    // allocations below (see ensure_ws)
    WISP_CUDA_TRY(cudaDeviceSynchronize());
    cudaPointerAttributes pa{};
    for (const void *hp : {host_w13, host_w2, fp8 ? host_s13 : host_w13, fp8 ? host_s2 : host_w2}) {
        if (cudaPointerGetAttributes(&pa, hp) != cudaSuccess || pa.type != cudaMemoryTypeHost) {
            cudaGetLastError();
            return fail(WISP_ERR_INVALID, "wisp_layer_create: host expert weights must be pinned");
        }
    }
    wisp_layer *L = new wisp_layer();
    L->dev = device;
    L->E = num_experts;
    L->cap = cap_experts;
    L->H = hidden;
    L->I = inter;
    L->mode = mode;
    L->b13 = w13_expert_bytes;
    L->b2 = w2_expert_bytes;
    L->h13 = reinterpret_cast<const char *>(host_w13);
    L->h2 = reinterpret_cast<const char *>(host_w2);
    if (fp8) {
        L->fp8 = true;
        L->bs13 = sizeof(float) * (2LL * inter / kFp8Block) * (hidden / kFp8Block);
        L->bs2 = sizeof(float) * (1LL * hidden / kFp8Block) * (inter / kFp8Block);
        L->hs13 = reinterpret_cast<const char *>(host_s13);
        L->hs2 = reinterpret_cast<const char *>(host_s2);
    }
    auto bail = [&](int rc) {
        wisp_layer_destroy(L);
        return rc;
    };
    if (alloc_slots(L, cap_experts))
        return bail(fail(WISP_ERR_NOMEM, "wisp_layer_create: HBM allocation failed"));
    if (cudaMalloc(&L->d_emap, sizeof(int32_t) * num_experts) != cudaSuccess ||
        cudaMalloc(&L->d_hdr, sizeof(int64_t) * 8) != cudaSuccess ||
        cudaMalloc(&L->d_bar, sizeof(unsigned int) * kBarWords) != cudaSuccess ||
        cudaMalloc(&L->d_last_unique, sizeof(uint32_t) * 32) != cudaSuccess ||
        cudaMalloc(&L->d_flow, sizeof(unsigned int) * kFlowWords) != cudaSuccess)
        return bail(fail(WISP_ERR_NOMEM, "wisp_layer_create: device allocation failed"));
    if (cudaMemset(L->d_emap, 0xff, sizeof(int32_t) * num_experts) != cudaSuccess ||
        cudaMemset(L->d_hdr, 0, sizeof(int64_t) * 8) != cudaSuccess ||
        cudaMemset(L->d_bar, 0, sizeof(unsigned int) * kBarWords) != cudaSuccess ||
        cudaMemset(L->d_last_unique, 0, sizeof(uint32_t) * 32) != cudaSuccess ||
        cudaMemset(L->d_flow, 0, sizeof(unsigned int) * kFlowWords) != cudaSuccess ||
        cudaHostAlloc(&L->h_done, sizeof(unsigned long long), cudaHostAllocMapped) != cudaSuccess ||
        cudaHostGetDevicePointer((void **)&L->d_done, L->h_done, 0) != cudaSuccess ||
        cudaHostAlloc(&L->h_status, sizeof(int32_t), cudaHostAllocMapped) != cudaSuccess ||
        cudaHostGetDevicePointer((void **)&L->d_status, L->h_status, 0) != cudaSuccess ||
        cudaHostAlloc(&L->h_flag_ring, sizeof(uint32_t) * kFlagRing, cudaHostAllocDefault) != cudaSuccess ||
        cudaStreamCreateWithFlags(&L->copy_stream, cudaStreamNonBlocking) != cudaSuccess ||
        cudaEventCreateWithFlags(&L->ev_pager, cudaEventDisableTiming) != cudaSuccess ||
        cudaEventCreateWithFlags(&L->ev_copies, cudaEventDisableTiming) != cudaSuccess ||
        cudaEventCreateWithFlags(&L->ev_last, cudaEventDisableTiming) != cudaSuccess ||
        cudaEventCreateWithFlags(&L->ev_pf, cudaEventDisableTiming) != cudaSuccess ||
        cudaHostAlloc(&L->h_pf, sizeof(int32_t) * ((size_t)num_experts + kMbRec * (num_experts + 1)),
                      cudaHostAllocMapped) != cudaSuccess ||
        cudaHostGetDevicePointer((void **)&L->d_pf, L->h_pf, 0) != cudaSuccess)
        return bail(fail(WISP_ERR_CUDA, "wisp_layer_create: buffer/stream/event setup failed"));
    *L->h_done = 0;
    *L->h_status = 0;
    for (auto &b : L->mb_busy) b.store(0);
    int rc = ensure_ws(L, 16, 8);
    if (rc) return bail(rc);
    if (cudaDeviceSynchronize() != cudaSuccess)
        return bail(fail(WISP_ERR_CUDA, "wisp_layer_create: device sync failed"));
    // One-launch forward by default only where it never waits on page-ins:
    // a paged forward's kernel would wait for copies a host thread issues
    // after the launch on another stream, and CUDA may queue those copies in a
    // hardware queue behind work the caller has already queued after the
    // kernel -- the kernel then waits until its limit.  WISP_CFG_ASYNC = 1
    // opts a paged layer in where the caller queues nothing on the device
    // while its forwards page in.
    L->async = (mode == WISP_MODE_RESIDENT) && !fp8;
    {
        int sms = 0;
        if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device) != cudaSuccess) sms = 0;
        L->tc_min_pairs = default_tc_min_pairs(hidden, inter, sms);
    }
    const char *env = getenv("WISP_B200_SYNC");
    if (env && env[0] == '1') L->async = false;
    *out = L;
    return WISP_OK;
}


extern "C" {

const char *wisp_version(void) { return "wisp_b200 0.2.0 (sm_100a)"; }

const char *wisp_last_error(void) { return g_last_error.c_str(); }

int wisp_layer_create(int32_t num_experts, int32_t cap_experts, int32_t hidden, int32_t inter,
                      int64_t w13_expert_bytes, int64_t w2_expert_bytes, const void *host_w13,
                      const void *host_w2, int32_t device, int32_t mode, wisp_layer **out) {
    return layer_create_impl(num_experts, cap_experts, hidden, inter, w13_expert_bytes, w2_expert_bytes,
                             host_w13, host_w2, device, mode, out);
}

int wisp_layer_create_fp8(int32_t num_experts, int32_t cap_experts, int32_t hidden, int32_t inter,
                          int32_t block_n, int32_t block_k, const void *host_w13, const void *host_w2,
                          const void *host_s13, const void *host_s2, int32_t device, int32_t mode,
                          wisp_layer **out) {
    if (!out) return fail(WISP_ERR_INVALID, "wisp_layer_create_fp8: out is NULL");
    *out = nullptr;
    if (block_n != kFp8Block || block_k != kFp8Block)
        return fail(WISP_ERR_UNSUPPORTED, "wisp_layer_create_fp8: weight blocks must be 128 x 128");
    if (hidden <= 0 || inter <= 0 || hidden % kFp8Block || inter % kFp8Block)
        return fail(WISP_ERR_UNSUPPORTED, "wisp_layer_create_fp8: hidden and inter must be multiples of 128");
    if (!host_s13 || !host_s2) return fail(WISP_ERR_INVALID, "wisp_layer_create_fp8: NULL scales");
    return layer_create_impl(num_experts, cap_experts, hidden, inter, 2LL * inter * hidden, 1LL * hidden * inter,
                             host_w13, host_w2, device, mode, out, host_s13, host_s2);
}

int wisp_layer_destroy(wisp_layer *L) {
    if (!L) return WISP_OK;
    DeviceGuard guard(L->dev);
    if (L->ev_last) drain(L);
    cudaDeviceSynchronize();
    free_ws(L);
    for (void *p : {(void *)L->d13, (void *)L->d2, (void *)L->ds13, (void *)L->ds2, (void *)L->d_s2e,
                    (void *)L->d_tick, (void *)L->d_emap,
                    (void *)L->d_hdr, (void *)L->d_slot_gen, (void *)L->d_slot_ready, (void *)L->d_bar,
                    (void *)L->d_flow, (void *)L->d_last_unique})
        cudaFree(p);
    if (L->h_done) cudaFreeHost(L->h_done);
    if (L->h_status) cudaFreeHost(L->h_status);
    if (L->h_flag_ring) cudaFreeHost(L->h_flag_ring);
    if (L->h_pf) cudaFreeHost(L->h_pf);
    if (L->ev_pf) cudaEventDestroy(L->ev_pf);
    for (auto e : L->ev_group) cudaEventDestroy(e);
    for (auto e : L->ev_copy) cudaEventDestroy(e);
    for (cudaEvent_t e : {L->ev_pager, L->ev_copies, L->ev_last})
        if (e) cudaEventDestroy(e);
    if (L->copy_stream) cudaStreamDestroy(L->copy_stream);
    delete L;
    return WISP_OK;
}

int wisp_moe_forward(wisp_layer *L, const void *x, const float *topk_weights,
                     const void *topk_ids, int32_t ids_int64, int32_t num_tokens, int32_t top_k,
                     void *out, void *stream) {
    if (!L) return fail(WISP_ERR_INVALID, "wisp_moe_forward: NULL layer");
    if (L->H <= 0 || L->I <= 0)
        return fail(WISP_ERR_UNSUPPORTED, "wisp_moe_forward: layer was created without a compute shape");
    if (num_tokens < 0 || top_k < 1 || top_k > 64)
        return fail(WISP_ERR_INVALID, "wisp_moe_forward: bad num_tokens/top_k");
    if (num_tokens > 0 && (!x || !topk_weights || !topk_ids || !out))
        return fail(WISP_ERR_INVALID, "wisp_moe_forward: NULL tensor");
    if (!aligned16(x) || !aligned16(out))
        return fail(WISP_ERR_INVALID, "wisp_moe_forward: x and out must be 16-byte aligned");
    std::lock_guard<std::mutex> lk(L->mu);
    DeviceGuard guard(L->dev);
    if (L->mode == WISP_MODE_RESIDENT && !L->primed && num_tokens > 0)
        return fail(WISP_ERR_INVALID,
                    "wisp_moe_forward: resident layer has no expert in its slots; call wisp_prime_identity first");
    int rc = take_errors(L);
    if (rc) return rc;
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    const Path path = compute_path(L, num_tokens, top_k);
    if (path == Path::kFp8) {  // FP8 layers: the host-synchronous path, every call size
        rc = run_pager(L, topk_ids, ids_int64, num_tokens, top_k, 0, 1, s);
        if (rc) return rc;
        return page_and_compute(L, x, topk_weights, num_tokens, top_k, out, s, true);
    }
    if (L->async && num_tokens > 0 && (path == Path::kBatchTC || path == Path::kPrefillTC) &&
        L->mode == WISP_MODE_RESIDENT)
        return forward_tc_resident(L, path, x, topk_weights, topk_ids, ids_int64, num_tokens, top_k, out, s);
    if (L->async && top_k <= L->cap && path == Path::kDecode)
        return forward_async(L, x, topk_weights, topk_ids, ids_int64, num_tokens, top_k, out, s);
    rc = run_pager(L, topk_ids, ids_int64, num_tokens, top_k, 0, 1, s);
    if (rc) return rc;
    return page_and_compute(L, x, topk_weights, num_tokens, top_k, out, s, true);
}

int wisp_ensure_resident(wisp_layer *L, const void *ids, int32_t ids_int64, int32_t n,
                         void *stream) {
    if (!L) return fail(WISP_ERR_INVALID, "wisp_ensure_resident: NULL layer");
    if (n < 0 || (n > 0 && !ids)) return fail(WISP_ERR_INVALID, "wisp_ensure_resident: bad ids");
    if (L->mode != WISP_MODE_PAGED)
        return fail(WISP_ERR_INVALID, "wisp_ensure_resident: layer is not in paged mode");
    std::lock_guard<std::mutex> lk(L->mu);
    DeviceGuard guard(L->dev);
    int rc = take_errors(L);
    if (rc) return rc;
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    rc = run_pager(L, ids, ids_int64, 1, n, 1, 0, s);
    if (rc) return rc;
    rc = page_and_compute(L, nullptr, nullptr, 1, n, nullptr, s, false);
    if (rc) return rc;
    WISP_CUDA_TRY(cudaStreamSynchronize(L->copy_stream));
    WISP_CUDA_TRY(cudaStreamSynchronize(s));
    return WISP_OK;
}

int wisp_pager_step(wisp_layer *L, const void *topk_ids, int32_t ids_int64, int32_t num_tokens,
                    int32_t top_k, int32_t *slots_out, void *stream) {
    if (!L) return fail(WISP_ERR_INVALID, "wisp_pager_step: NULL layer");
    if (num_tokens < 0 || top_k < 1 || (num_tokens > 0 && !topk_ids))
        return fail(WISP_ERR_INVALID, "wisp_pager_step: bad ids");
    std::lock_guard<std::mutex> lk(L->mu);
    DeviceGuard guard(L->dev);
    int rc = take_errors(L);
    if (rc) return rc;
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    rc = run_pager(L, topk_ids, ids_int64, num_tokens, top_k, 0, 1, s);
    if (rc) return rc;
    rc = page_and_compute(L, nullptr, nullptr, num_tokens, top_k, nullptr, s, false);
    if (rc) return rc;
    WISP_CUDA_TRY(cudaStreamSynchronize(L->copy_stream));
    WISP_CUDA_TRY(cudaStreamSynchronize(s));
    if (slots_out && num_tokens > 0)
        WISP_CUDA_TRY(cudaMemcpy(slots_out, L->d_slots, sizeof(int32_t) * (size_t)num_tokens * top_k,
                                 cudaMemcpyDeviceToHost));
    return WISP_OK;
}

int wisp_prefetch_async(wisp_layer *L, const int32_t *predicted, int32_t n, void *stream) {
    if (!L) return fail(WISP_ERR_INVALID, "wisp_prefetch_async: NULL layer");
    if (n < 0 || n > L->E || (n > 0 && !predicted))
        return fail(WISP_ERR_INVALID, "wisp_prefetch_async: n must be in [0, num_experts]");
    if (L->mode != WISP_MODE_PAGED) return fail(WISP_ERR_INVALID, "wisp_prefetch_async: layer is not paged");
    (void)stream;
    std::lock_guard<std::mutex> lk(L->mu);
    DeviceGuard guard(L->dev);
    int rc = take_errors(L);
    if (rc) return rc;
    if (n == 0) return WISP_OK;
    std::copy(predicted, predicted + n, L->h_pf);
    int32_t *out = L->h_pf + L->E;
    out[0] = -1;
    PrefetchParams p{};
    p.pred = L->d_pf;
    p.n = n;
    p.E = L->E;
    p.cap = L->cap;
    p.s2e = L->d_s2e;
    p.tick = L->d_tick;
    p.emap = L->d_emap;
    p.hdr = L->d_hdr;
    p.slot_gen = L->d_slot_gen;
    p.last_unique = L->d_last_unique;
    p.out = L->d_pf + L->E;
    // on the copy stream, after this layer's last forward is done with its
    // slots and state; the next forward's pager waits for these copies
    WISP_CUDA_TRY(cudaStreamWaitEvent(L->copy_stream, L->ev_last, 0));
    rc = launch_prefetch(p, L->copy_stream);
    if (rc) return rc;
    ++L->launches;
    WISP_CUDA_TRY(cudaEventRecord(L->ev_pf, L->copy_stream));
    WISP_CUDA_TRY(cudaEventSynchronize(L->ev_pf));
    const volatile int32_t *vo = out;
    if (vo[0] == WISP_ERR_BAD_EXPERT)
        return fail(WISP_ERR_BAD_EXPERT, "wisp_prefetch_async: predicted id outside [0, " + std::to_string(L->E) + ")");
    if (vo[0] != WISP_OK) return fail(WISP_ERR_CUDA, "wisp_prefetch_async: prefetch kernel did not report");
    const int nload = vo[1];
    for (int i = 0; i < nload; ++i) {
        const volatile int32_t *r = out + kMbRec * (i + 1);
        rc = issue_pagein(L, r[0], r[1], (uint32_t)r[2]);
        if (rc) return rc;
    }
    WISP_CUDA_TRY(cudaEventRecord(L->ev_copies, L->copy_stream));
    ++L->copy_gen;
    return WISP_OK;
}

int wisp_prime_identity(wisp_layer *L, void *stream) {
    if (!L) return fail(WISP_ERR_INVALID, "wisp_prime_identity: NULL layer");
    if (L->cap != L->E) return fail(WISP_ERR_INVALID, "prime_identity requires cap == num_experts");
    std::lock_guard<std::mutex> lk(L->mu);
    DeviceGuard guard(L->dev);
    int rc = drain(L);
    if (rc) return rc;
    std::vector<int32_t> ident(L->E);
    for (int i = 0; i < L->E; ++i) ident[i] = i;
    // the copy stream carries copies and flag writes only (no kernels)
    WISP_CUDA_TRY(cudaMemcpyAsync(L->d13, L->h13, (size_t)L->E * L->b13, cudaMemcpyHostToDevice,
                                  L->copy_stream));
    WISP_CUDA_TRY(cudaMemcpyAsync(L->d2, L->h2, (size_t)L->E * L->b2, cudaMemcpyHostToDevice,
                                  L->copy_stream));
    if (L->fp8) {
        WISP_CUDA_TRY(cudaMemcpyAsync(L->ds13, L->hs13, (size_t)L->E * L->bs13, cudaMemcpyHostToDevice,
                                      L->copy_stream));
        WISP_CUDA_TRY(cudaMemcpyAsync(L->ds2, L->hs2, (size_t)L->E * L->bs2, cudaMemcpyHostToDevice,
                                      L->copy_stream));
    }
    WISP_CUDA_TRY(cudaMemcpy(L->d_s2e, ident.data(), sizeof(int32_t) * L->E, cudaMemcpyHostToDevice));
    WISP_CUDA_TRY(cudaMemcpy(L->d_emap, ident.data(), sizeof(int32_t) * L->E, cudaMemcpyHostToDevice));
    WISP_CUDA_TRY(cudaMemcpy(L->d_slot_ready, L->d_slot_gen, sizeof(uint32_t) * L->cap,
                             cudaMemcpyDeviceToDevice));
    WISP_CUDA_TRY(cudaEventRecord(L->ev_copies, L->copy_stream));
    ++L->copy_gen;
    WISP_CUDA_TRY(cudaStreamWaitEvent(reinterpret_cast<cudaStream_t>(stream), L->ev_copies, 0));
    L->primed = true;
    return WISP_OK;
}

int wisp_resize_cap(wisp_layer *L, int32_t new_cap, void *stream) {
    if (!L) return fail(WISP_ERR_INVALID, "wisp_resize_cap: NULL layer");
    (void)stream;
    std::lock_guard<std::mutex> lk(L->mu);
    DeviceGuard guard(L->dev);
    if (L->mode != WISP_MODE_PAGED) return fail(WISP_ERR_INVALID, "wisp_resize_cap: not a paged layer");
    new_cap = std::max(2, std::min((int)new_cap, L->E));
    if (new_cap == L->cap) return WISP_OK;
    int rc = drain(L);
    if (rc) return rc;
    WISP_CUDA_TRY(cudaDeviceSynchronize());  // drained barrier, as the reference requires
    const int old = L->cap, keep = std::min(old, new_cap);
    std::vector<int32_t> s2e(old), emap(L->E);
    std::vector<int64_t> tick(old);
    std::vector<uint32_t> gen(old);
    WISP_CUDA_TRY(cudaMemcpy(s2e.data(), L->d_s2e, sizeof(int32_t) * old, cudaMemcpyDeviceToHost));
    WISP_CUDA_TRY(cudaMemcpy(tick.data(), L->d_tick, sizeof(int64_t) * old, cudaMemcpyDeviceToHost));
    WISP_CUDA_TRY(cudaMemcpy(emap.data(), L->d_emap, sizeof(int32_t) * L->E, cudaMemcpyDeviceToHost));
    WISP_CUDA_TRY(cudaMemcpy(gen.data(), L->d_slot_gen, sizeof(uint32_t) * old, cudaMemcpyDeviceToHost));
    char *o13 = L->d13, *o2 = L->d2, *os13 = L->ds13, *os2 = L->ds2;
    int32_t *os2e = L->d_s2e;
    int64_t *otick = L->d_tick;
    uint32_t *ogen = L->d_slot_gen, *oready = L->d_slot_ready;
    L->d13 = L->d2 = L->ds13 = L->ds2 = nullptr;
    if (alloc_slots(L, new_cap)) {
        for (void *p : {(void *)L->d13, (void *)L->d2, (void *)L->ds13, (void *)L->ds2, (void *)L->d_s2e,
                        (void *)L->d_tick, (void *)L->d_slot_gen, (void *)L->d_slot_ready})
            cudaFree(p);
        L->d13 = o13;
        L->d2 = o2;
        L->ds13 = os13;
        L->ds2 = os2;
        L->d_s2e = os2e;
        L->d_tick = otick;
        L->d_slot_gen = ogen;
        L->d_slot_ready = oready;
        return fail(WISP_ERR_NOMEM, "wisp_resize_cap: HBM allocation failed");
    }
    WISP_CUDA_TRY(cudaMemcpy(L->d13, o13, (size_t)keep * L->b13, cudaMemcpyDeviceToDevice));
    WISP_CUDA_TRY(cudaMemcpy(L->d2, o2, (size_t)keep * L->b2, cudaMemcpyDeviceToDevice));
    if (L->fp8) {
        WISP_CUDA_TRY(cudaMemcpy(L->ds13, os13, (size_t)keep * L->bs13, cudaMemcpyDeviceToDevice));
        WISP_CUDA_TRY(cudaMemcpy(L->ds2, os2, (size_t)keep * L->bs2, cudaMemcpyDeviceToDevice));
    }
    if (new_cap < old)
        for (int s = new_cap; s < old; ++s)
            if (s2e[s] >= 0) emap[s2e[s]] = -1;
    s2e.resize(new_cap, -1);
    tick.resize(new_cap, 0);
    gen.resize(new_cap, 0);
    WISP_CUDA_TRY(cudaMemcpy(L->d_s2e, s2e.data(), sizeof(int32_t) * new_cap, cudaMemcpyHostToDevice));
    WISP_CUDA_TRY(cudaMemcpy(L->d_tick, tick.data(), sizeof(int64_t) * new_cap, cudaMemcpyHostToDevice));
    WISP_CUDA_TRY(cudaMemcpy(L->d_emap, emap.data(), sizeof(int32_t) * L->E, cudaMemcpyHostToDevice));
    // every copy has landed at this barrier: generation flags equal the generations
    WISP_CUDA_TRY(cudaMemcpy(L->d_slot_gen, gen.data(), sizeof(uint32_t) * new_cap, cudaMemcpyHostToDevice));
    WISP_CUDA_TRY(cudaMemcpy(L->d_slot_ready, gen.data(), sizeof(uint32_t) * new_cap, cudaMemcpyHostToDevice));
    for (void *p : {(void *)o13, (void *)o2, (void *)os13, (void *)os2, (void *)os2e, (void *)otick, (void *)ogen,
                    (void *)oready})
        if (p) cudaFree(p);
    L->cap = new_cap;
    return WISP_OK;
}

int wisp_get_state(wisp_layer *L, int32_t *slot_to_expert, int64_t *lru_tick, int64_t *clock,
                   int64_t *stats4, int32_t *expert_map, int32_t *cap) {
    if (!L) return fail(WISP_ERR_INVALID, "wisp_get_state: NULL layer");
    std::lock_guard<std::mutex> lk(L->mu);
    DeviceGuard guard(L->dev);
    WISP_CUDA_TRY(cudaDeviceSynchronize());
    if (cap) *cap = L->cap;
    if (slot_to_expert)
        WISP_CUDA_TRY(cudaMemcpy(slot_to_expert, L->d_s2e, sizeof(int32_t) * L->cap, cudaMemcpyDeviceToHost));
    if (lru_tick)
        WISP_CUDA_TRY(cudaMemcpy(lru_tick, L->d_tick, sizeof(int64_t) * L->cap, cudaMemcpyDeviceToHost));
    if (expert_map)
        WISP_CUDA_TRY(cudaMemcpy(expert_map, L->d_emap, sizeof(int32_t) * L->E, cudaMemcpyDeviceToHost));
    int64_t hdr[5];
    WISP_CUDA_TRY(cudaMemcpy(hdr, L->d_hdr, sizeof(hdr), cudaMemcpyDeviceToHost));
    if (clock) *clock = hdr[0];
    if (stats4)
        for (int i = 0; i < 4; ++i) stats4[i] = hdr[1 + i];
    return WISP_OK;
}

int wisp_set_stats(wisp_layer *L, const int64_t *stats4) {
    if (!L || !stats4) return fail(WISP_ERR_INVALID, "wisp_set_stats: NULL argument");
    std::lock_guard<std::mutex> lk(L->mu);
    DeviceGuard guard(L->dev);
    WISP_CUDA_TRY(cudaDeviceSynchronize());
    WISP_CUDA_TRY(cudaMemcpy(L->d_hdr + 1, stats4, sizeof(int64_t) * 4, cudaMemcpyHostToDevice));
    return WISP_OK;
}

int wisp_layer_buffers(wisp_layer *L, void **scratch_w13, void **scratch_w2, void **expert_map) {
    if (!L) return fail(WISP_ERR_INVALID, "wisp_layer_buffers: NULL layer");
    if (scratch_w13) *scratch_w13 = L->d13;
    if (scratch_w2) *scratch_w2 = L->d2;
    if (expert_map) *expert_map = L->d_emap;
    return WISP_OK;
}

int wisp_layer_scale_buffers(wisp_layer *L, void **scratch_s13, void **scratch_s2) {
    if (!L) return fail(WISP_ERR_INVALID, "wisp_layer_scale_buffers: NULL layer");
    if (!L->fp8) return fail(WISP_ERR_INVALID, "wisp_layer_scale_buffers: not an FP8 layer");
    if (scratch_s13) *scratch_s13 = L->ds13;
    if (scratch_s2) *scratch_s2 = L->ds2;
    return WISP_OK;
}

int wisp_get_telemetry(wisp_layer *L, int64_t *out4) {
    if (!L || !out4) return fail(WISP_ERR_INVALID, "wisp_get_telemetry: NULL argument");
    std::lock_guard<std::mutex> lk(L->mu);
    DeviceGuard guard(L->dev);
    WISP_CUDA_TRY(cudaDeviceSynchronize());
    int64_t hdr[7];
    WISP_CUDA_TRY(cudaMemcpy(hdr, L->d_hdr, sizeof(hdr), cudaMemcpyDeviceToHost));
    out4[0] = hdr[5];
    out4[1] = hdr[2];
    out4[2] = hdr[2] * (L->b13 + L->b2);
    out4[3] = hdr[6];
    return WISP_OK;
}

int wisp_get_last_unique_experts(wisp_layer *L, int32_t *ids_out, int32_t max_ids, int32_t *n_out) {
    if (!L || !n_out || max_ids < 0 || (max_ids > 0 && !ids_out))
        return fail(WISP_ERR_INVALID, "wisp_get_last_unique_experts: bad argument");
    std::lock_guard<std::mutex> lk(L->mu);
    DeviceGuard guard(L->dev);
    uint32_t words[32];
    if (L->last_unique_host) {
        std::copy(L->h_last_unique, L->h_last_unique + 32, words);
    } else {
        WISP_CUDA_TRY(cudaDeviceSynchronize());
        WISP_CUDA_TRY(cudaMemcpy(words, L->d_last_unique, sizeof(words), cudaMemcpyDeviceToHost));
    }
    int n = 0;
    for (int e = 0; e < L->E; ++e)
        if ((words[e >> 5] >> (e & 31)) & 1u) {
            if (n < max_ids) ids_out[n] = e;
            ++n;
        }
    *n_out = n;
    return WISP_OK;
}

int wisp_get_launch_count(wisp_layer *L, int64_t *out) {
    if (!L || !out) return fail(WISP_ERR_INVALID, "wisp_get_launch_count: NULL argument");
    std::lock_guard<std::mutex> lk(L->mu);
    *out = L->launches;
    return WISP_OK;
}

int wisp_layer_sync(wisp_layer *L) {
    if (!L) return fail(WISP_ERR_INVALID, "wisp_layer_sync: NULL layer");
    std::lock_guard<std::mutex> lk(L->mu);
    DeviceGuard guard(L->dev);
    int rc = drain(L);
    if (rc) return rc;
    return take_errors(L);
}

int wisp_layer_query(wisp_layer *L, int32_t key, int64_t *value) {
    if (!L || !value) return fail(WISP_ERR_INVALID, "wisp_layer_query: NULL argument");
    std::lock_guard<std::mutex> lk(L->mu);
    switch (key) {
        case WISP_CFG_ASYNC:
            *value = L->async ? 1 : 0;
            return WISP_OK;
        case WISP_CFG_WAIT_NS:
            *value = L->wait_ns;
            return WISP_OK;
        case WISP_CFG_TC_MIN_PAIRS:
            *value = L->tc_min_pairs;
            return WISP_OK;
        case WISP_CFG_COMPUTE_CLASS:
            *value = L->compute_class;
            return WISP_OK;
        default:
            return fail(WISP_ERR_INVALID, "wisp_layer_query: unknown key");
    }
}

int wisp_layer_reserve(wisp_layer *L, int32_t num_tokens, int32_t top_k) {
    if (!L) return fail(WISP_ERR_INVALID, "wisp_layer_reserve: NULL layer");
    if (num_tokens < 0 || top_k < 1) return fail(WISP_ERR_INVALID, "wisp_layer_reserve: bad sizes");
    std::lock_guard<std::mutex> lk(L->mu);
    if (num_tokens <= L->wsT && top_k <= L->wsK) return WISP_OK;
    DeviceGuard guard(L->dev);
    int rc = drain(L);
    if (rc) return rc;
    return ensure_ws(L, num_tokens, top_k);
}

int wisp_layer_config(wisp_layer *L, int32_t key, int64_t value) {
    if (!L) return fail(WISP_ERR_INVALID, "wisp_layer_config: NULL layer");
    std::lock_guard<std::mutex> lk(L->mu);
    switch (key) {
        case WISP_CFG_ASYNC:
            L->async = value != 0;
            return WISP_OK;
        case WISP_CFG_WAIT_NS:
            if (value < 1000000) return fail(WISP_ERR_INVALID, "wisp_layer_config: wait limit below 1 ms");
            L->wait_ns = value;
            return WISP_OK;
        case WISP_CFG_DROP_PAGEINS:
            L->drop_pageins.store((int)std::max<int64_t>(value, 0));
            return WISP_OK;
        case WISP_CFG_TRACE_BUFFER:
            L->trace = reinterpret_cast<unsigned long long *>(value);
            return WISP_OK;
        case WISP_CFG_TC_MIN_PAIRS:
            if (value < 1) return fail(WISP_ERR_INVALID, "wisp_layer_config: tensor-core threshold below 1 pair");
            L->tc_min_pairs = (int)std::min<int64_t>(value, kPrefillMinPairs);
            return WISP_OK;
        case WISP_CFG_COMPUTE_CLASS:
            if (value < 0 || value > 2) return fail(WISP_ERR_INVALID, "wisp_layer_config: compute class 0, 1 or 2");
            L->compute_class = (int)value;
            return WISP_OK;
        default:
            return fail(WISP_ERR_INVALID, "wisp_layer_config: unknown key");
    }
}

}  // extern "C"
