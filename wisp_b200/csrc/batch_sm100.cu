// Decode-batch expert compute on tcgen05 tensor cores, weight-stationary.
//
// In a decode batch an expert sees a handful of tokens, so the token-major
// tiles of the prefill GEMMs (128 pairs on the MMA's M side) would spend the
// tensor cores on padding rows.  Here the weights take the M side and the
// tokens the N side, so the tensor work is 32 token columns per weight row
// and the path is bound by streaming the weights from HBM:
//
//   gate-up  tile (token block b of expert u, 128 intermediate rows j):
//            G[128 x 32] = W13 rows j . X_perm rows^T and
//            U[128 x 32] = W13 rows I + j . X_perm rows^T over K = H: two MMAs
//            (M 128, N 32, K 16) per K step on the same token tile; thread
//            (TMEM lane) r holds g and u of intermediate row j + r for the
//            block's tokens and stores act_perm[q][j + r] =
//            bf16(bf16(silu(bf16(g))) * bf16(u));
//   down     tile (token block b, 256 hidden rows h):
//            Y0 / Y1 [128 x 32] = W2 rows h / h + 128 . act_perm rows^T over
//            K = I; y[pair][h + r] = bf16(acc * routing weight).
//
// A token block is up to 32 consecutive rows of one expert in the call's
// expert-major pair order, so each weight tile is streamed once per token
// block, i.e. once per expert for a decode batch.  Gate-up and down share ONE
// persistent launch: tiles are numbered gate-up first, then down, both in
// token-block order, handed out in that order by a per-launch counter: each
// CTA's producer takes the next index when it starts a tile and passes it to
// the MMA thread and the epilogue through a small shared-memory ring, so
// CTAs that drew heavy tiles take fewer (dynamic balance; a down tile's
// gate-up tiles were always taken earlier, by running CTAs).  Before the
// producer loads a down tile it
// waits until the block's gate-up tiles have published their activation rows:
// every epilogue warp adds 1 to the block's counter after its stores (release
// at GPU scope, after an async-proxy fence, since the rows are read back by
// TMA), and the producer waits for 4 * I / 128 (acquire, then an async-proxy
// fence).  Gate-up tiles wait for nothing, and the launch is cooperative
// (every CTA resident), so these waits end; each is bounded all the same and
// a CTA that gives up raises a device-wide abort word that ends the others'
// waits.  The counters come in two halves by launch parity: a launch uses one
// and zeroes the other for the next launch.
//
// The expert lists come either from the pager (paged layers: u_off / u_pairs
// / u_slot in global memory, X_perm written by the gather kernel) or, for a
// resident layer's call, from the kernel itself: every CTA sorts the call's
// (at most 512) pairs by expert in shared memory -- experts ascending, pairs
// ascending within an expert, slots from the expert map -- copies every
// gridDim.x-th row of X_perm (its share) and counts itself in; a producer
// waits for all CTAs' shares before its first gate-up load.
//
// Roles per CTA (192 threads, one CTA per SM): warp 0 lane 0 issues the TMA
// loads of a 6-stage ring (two 128 x 64 weight boxes and one 32 x 64 token
// box per stage, 128-byte swizzle, weights with an L2 evict-first hint as
// they are read once); warp 1 lane 0 issues the MMAs into one of two
// 64-column TMEM accumulators; warps 2..5 read an accumulator back with
// tcgen05.ld (warp w owns TMEM lanes 32 (w % 4) ..) while the next tile
// accumulates into the other.
//
// Each output element is its own dot product with the K blocks in order, so
// results do not depend on which tokens or experts share a tile, the slots,
// the cap or the grouping; they are byte-identical to the token-major GEMMs'.
#include "gemm_sm100.cuh"
#include "prefill.cuh"

#include <algorithm>

namespace wisp {
namespace batch {
namespace {

using gemm::mbar_arrive;
using gemm::mbar_expect_tx;
using gemm::mbar_init;
using gemm::mbar_wait;
using gemm::s_addr;
using gemm::smem_desc_k_sw128;
using gemm::tc_fence_after;
using gemm::tc_fence_before;
using gemm::tma_load_2d;
using gemm::tma_load_2d_hint;
using gemm::tmem_alloc;
using gemm::tmem_dealloc;
using gemm::tmem_ld32;
using gemm::umma_commit;
using gemm::umma_f16;

constexpr int kWM = 128;                          // weight rows per MMA (M): TMEM lanes
constexpr int kTN = kBatchTokens;                 // token rows per tile (N)
constexpr int kBK = 64;                           // K per stage: one 128-byte swizzle row
constexpr int kStages = 6;
constexpr int kThreads = 192;                     // producer warp, MMA warp, 4 epilogue warps
constexpr int kEpiThreads = 128;
constexpr int kEpiWarps = kEpiThreads / 32;
constexpr int kWBoxBytes = kWM * kBK * 2;         // 16 KB
constexpr int kTBoxBytes = kTN * kBK * 2;         // 4 KB
constexpr int kStageBytes = 2 * kWBoxBytes + kTBoxBytes;
constexpr int kSmemBytes = kStages * kStageBytes + 1024;  // + slack to align stages to 1024 B
constexpr int kAccCols = 2 * kTN;                 // one tile: two accumulators of kTN columns
constexpr int kTmemCols = 2 * kAccCols;           // double-buffered
constexpr int kDownRows = 2 * kWM;                // hidden rows per down tile
constexpr int kMaxPairs = kBatchMaxPairs;
constexpr int kMaxRouteExperts = 1024;
static_assert(kTmemCols >= 32 && (kTmemCols & (kTmemCols - 1)) == 0, "TMEM allocation: power of two >= 32");
static_assert(kTN == 32, "the epilogue reads one 32-column TMEM block per accumulator");
static_assert(3 * kMaxRouteExperts * 4 + kMaxPairs * 4 <= kStages * kStageBytes, "routing scratch fits the ring");
static_assert(kMaxPairs + (kMaxPairs + kTN - 1) / kTN + 3 == kBatchReadyWords, "counter words");
constexpr int kTileRing = 4;                      // tile indices handed from the producer to the other roles
constexpr int kMaxBlocks = kMaxPairs + (kMaxPairs + kTN - 1) / kTN;

struct Args {
    // lists from the pager (route == false)
    const int32_t *u_off;       // [nu + 1]
    const int32_t *u_pairs;     // [npairs] absolute pair index, expert-major
    const int32_t *u_slot;      // [nu]
    const int32_t *nu_dev;
    const int32_t *pager_status;
    const int32_t *u_gen;       // [nu] generation each expert's slot must reach before its loads, or nullptr
    const uint32_t *slot_ready; // [slots] generation landed in each slot
    // in-kernel routing (route == true)
    int route;
    const void *ids;
    int ids64, T, K, E, count_forward;
    const int32_t *emap;
    const uint4 *x;             // [T][H / 8]
    uint4 *x_perm;              // [npairs][H / 8]
    int64_t *hdr;
    int32_t *dev_status;
    // both
    int H, I, Kc, t0;           // Kc: top-k; t0: first token of the group
    const float *topk_w;        // [T * K]
    __nv_bfloat16 *act_perm;    // [npairs][I]
    __nv_bfloat16 *y;           // [T * K][H]
    __nv_bfloat16 *out;         // [T][H]
    uint32_t *ready;            // this launch's counters: [blocks], gathered CTAs, abort word
    uint32_t *ready_next;       // the other half, zeroed for the next launch
    uint32_t *done;             // [tokens][H / 256][4] down rows stored, per epilogue warp
    uint32_t *done_next;        // the other half, zeroed for the next launch
    int *status;
    long long wait_ns;
    unsigned long long *trace;  // debug: per CTA kTraceWords %globaltimer milestones, or nullptr
};

// Trace milestones of a CTA (words 8 + kTraceWords * blockIdx.x + i).
enum { kTrEntry, kTrLists, kTrRoles, kTrFirstLoad, kTrLastLoad, kTrLastMma, kTrEpiDone, kTrExit, kTraceWords };
__device__ __forceinline__ void trace_at(const unsigned long long *tr, int i) {
    if (tr) const_cast<unsigned long long *>(tr)[8 + kTraceWords * blockIdx.x + i] = globaltimer_ns();
}

struct Ring {
    uint64_t full[kStages], empty[kStages];
    uint64_t acc_full[2], acc_empty[2], mma_done;
    uint64_t tile_full[kTileRing], tile_empty[kTileRing];
    int tile[kTileRing];  // i-th tile of this CTA at [i % kTileRing]; -1: no more
    uint32_t tmem_base;
    int abort;
    int issued, consumed;
};

// The MMA thread's and the epilogue warps' i-th tile (bounded wait; -1 when
// there are no more or the wait gave up).  The epilogue's lane 0 and the MMA
// thread release the entry.
__device__ __forceinline__ int next_tile(Ring &R, int i, const Args &g, bool release) {
    volatile int *abort = &R.abort;
    const int slot = i % kTileRing;
    if (!mbar_wait(&R.tile_full[slot], (i / kTileRing) & 1, g.wait_ns, abort)) return -1;
    const int t = *reinterpret_cast<volatile int *>(&R.tile[slot]);
    if (release) mbar_arrive(&R.tile_empty[slot]);
    return t;
}

// The call's (or group's) experts, their token blocks and pair lists.
// Index arrays are 16-bit (offsets <= 512, blocks <= 528, slots < 1024) so
// that 512 pairs' lists fit beside the 6-stage ring.
struct Lists {
    int nu, nblocks, bad;
    int pairs[kMaxPairs];          // routed lists: absolute pair index, expert-major
    int16_t off[kMaxPairs + 1];    // pair-list offsets
    int16_t first[kMaxPairs + 1];  // first token block of each expert (prefix of block counts)
    int16_t slot[kMaxPairs];       // slot of each expert
    int16_t rows[kMaxBlocks];      // rows of each token block
    int16_t order[kMaxBlocks];     // blocks by rows, most first (ties: lower block first)
};
static_assert(kMaxPairs + 1 <= 32767 && kMaxBlocks <= 32767 && kMaxRouteExperts <= 32767, "16-bit lists");

// Token block b -> expert u, first list position q0, rows.
__device__ __forceinline__ void block_of(const Lists &L, int b, int &u, int &q0, int &rows) {
    int lo = 0, hi = L.nu - 1;
    while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (L.first[mid] <= b)
            lo = mid;
        else
            hi = mid - 1;
    }
    u = lo;
    q0 = L.off[u] + (b - L.first[u]) * kTN;
    rows = min(kTN, L.off[u + 1] - q0);
}

struct Tile {
    int down;  // 0: gate-up, 1: down
    int b;     // token block
    int col;   // 128-row block of I (gate-up) or 256-row block of H (down)
};
// Tiles in block order (blocks with the most rows first): the epilogue
// work of a tile grows with its rows and the combines of a token fall to its
// last tile, so the last tiles handed out are the lightest.
__device__ __forceinline__ Tile tile_at(const Lists &L, int t, int ngu, int cj, int ch) {
    if (t < ngu) return Tile{0, L.order[t / cj], t % cj};
    t -= ngu;
    return Tile{1, L.order[t / ch], t % ch};
}

__device__ __forceinline__ uint64_t policy_evict_first() {
    uint64_t pol;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
    return pol;
}
__device__ __forceinline__ void fence_proxy_async_global() {
    asm volatile("fence.proxy.async.global;" ::: "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_gpu(const uint32_t *p) {
    uint32_t v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void red_release_gpu_add(uint32_t *p, uint32_t v) {
    asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t atom_add_acq_rel_gpu(uint32_t *p, uint32_t v) {
    uint32_t old;
    asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
    return old;
}

constexpr int kGatheredWord = kBatchReadyWords - 3;
constexpr int kSchedWord = kBatchReadyWords - 2;
constexpr int kAbortWord = kBatchReadyWords - 1;

__device__ __forceinline__ void give_up(Ring &R, const Args &g) {
    R.abort = 1;
    if (g.status) *reinterpret_cast<volatile int *>(g.status) = WISP_ERR_TIMEOUT;
    atomicExch(g.ready + kAbortWord, 1u);  // ends the other CTAs' waits
}

// Producer wait on a counter word of this launch (a down tile's block: its
// activation rows published; kGatheredWord: every CTA's X_perm rows).
__device__ __forceinline__ bool wait_ready(const Args &g, int word_index, uint32_t need, volatile int *abort) {
    const uint32_t *word = g.ready + word_index;
    const volatile uint32_t *abort_all = g.ready + kAbortWord;
    if (ld_acquire_gpu(word) < need) {
        const unsigned long long t0 = globaltimer_ns();
        while (ld_acquire_gpu(word) < need) {
            if (*abort || *abort_all) return false;
            if ((long long)(globaltimer_ns() - t0) > g.wait_ns) return false;
            __nanosleep(32);
        }
    }
    fence_proxy_async_global();  // the rows (generic-proxy stores) before the TMA reads
    return true;
}

// Producer wait until expert u's slot holds the generation its page-in
// writes (the copy stream raises slot_ready after the copies).
__device__ __forceinline__ bool wait_slot(const Args &g, int u, int slot, volatile int *abort) {
    const uint32_t need = (uint32_t)g.u_gen[u];
    if (need == 0) return true;
    const uint32_t *word = g.slot_ready + slot;
    const volatile uint32_t *abort_all = g.ready + kAbortWord;
    if (ld_acquire_gpu(word) < need) {
        const unsigned long long t0 = globaltimer_ns();
        while (ld_acquire_gpu(word) < need) {
            if (*abort || *abort_all) return false;
            if ((long long)(globaltimer_ns() - t0) > g.wait_ns) return false;
            __nanosleep(64);
        }
    }
    fence_proxy_async_global();  // the copy engine's writes before the TMA reads
    return true;
}

__device__ __forceinline__ unsigned char *align1024(unsigned char *p) {
    const uint32_t a = s_addr(p);
    return p + ((1024u - (a & 1023u)) & 1023u);
}

// After an epilogue warp stored its rows h and h + 128 of a down tile's
// pairs: count the warp in for each of those pairs' tokens (lane n takes row
// n, all rows at once, acquire-release at GPU scope after a warp barrier, so
// the other lanes' stores are released too); the warp that brings a (token,
// 256-row block, quarter) counter to top-k holds the last of the token's
// weighted rows there and writes out[t] = the routing-order sum of the bf16
// rows y[t * K + k] (combine_add), rounded to bf16 (the combine kernel's
// arithmetic), loading up to 8 rows at a time past L1 before summing them.
__device__ __forceinline__ void combine_rows(const Args &g, const int32_t *pairs, int q0, int rows, int col,
                                             int quarter, int lane, int h) {
    const int K = g.Kc, H = g.H, ch = H / kDownRows;
    __syncwarp();
    int t = 0;
    bool last = false;
    if (lane < rows) {
        t = pairs[q0 + lane] / K;
        last = atom_add_acq_rel_gpu(g.done + ((size_t)(t - g.t0) * ch + col) * 4 + quarter, 1u) + 1 == (uint32_t)K;
    }
    unsigned lm = __ballot_sync(0xffffffffu, last);
    __syncwarp();
    while (lm) {
        const int n = __ffs(lm) - 1;
        lm &= lm - 1;
        const int tt = __shfl_sync(0xffffffffu, t, n);
        const unsigned short *row = reinterpret_cast<const unsigned short *>(g.y + (size_t)tt * K * H + h);
        float a0 = 0.f, a1 = 0.f;
        for (int k0 = 0; k0 < K; k0 += 8) {
            unsigned short v0[8], v1[8];
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                if (k0 + j < K) {
                    v0[j] = __ldcg(row + (size_t)(k0 + j) * H);
                    v1[j] = __ldcg(row + (size_t)(k0 + j) * H + kWM);
                }
            }
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                if (k0 + j < K) {
                    a0 = combine_add(a0, bf16lo((uint32_t)v0[j]), K);
                    a1 = combine_add(a1, bf16lo((uint32_t)v1[j]), K);
                }
            }
        }
        g.out[(size_t)tt * H + h] = __float2bfloat16_rn(a0);
        g.out[(size_t)tt * H + h + kWM] = __float2bfloat16_rn(a1);
    }
}

// Every CTA: the call's pairs sorted by expert (experts ascending, pairs
// ascending within one), with the ring as scratch.  Sets L.bad on an id
// outside [0, E).
__device__ void route_pairs(const Args &g, Lists &L, unsigned char *scratch) {
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int E = g.E, P = g.T * g.K;
    int *cnt = reinterpret_cast<int *>(scratch);  // [E] pairs per expert
    int *base = cnt + kMaxRouteExperts;           // [E] next list position of each expert
    int *emap = base + kMaxRouteExperts;          // [E] slot of each expert
    int *ids = emap + kMaxRouteExperts;           // [P]
    // the ids (at most 3 per thread: P <= 512 <= 3 * kThreads) and the map in flight together
    constexpr int kIdsPerThread = (kMaxPairs + kThreads - 1) / kThreads;
    long long v[kIdsPerThread];
#pragma unroll
    for (int j = 0; j < kIdsPerThread; ++j) {
        const int p = tid + j * kThreads;
        v[j] = p >= P ? 0
                      : g.ids64 ? reinterpret_cast<const int64_t *>(g.ids)[p]
                                : (long long)reinterpret_cast<const int32_t *>(g.ids)[p];
    }
    for (int e = tid; e < E; e += blockDim.x) {
        cnt[e] = 0;
        emap[e] = g.emap[e];
    }
    __syncthreads();
    bool bad = false;
#pragma unroll
    for (int j = 0; j < kIdsPerThread; ++j) {
        const int p = tid + j * kThreads;
        if (p < P) {
            const bool ok = v[j] >= 0 && v[j] < E;
            bad |= !ok;
            ids[p] = ok ? (int)v[j] : 0;
            if (ok) atomicAdd(&cnt[(int)v[j]], 1);
        }
    }
    if (__syncthreads_or(bad)) {
        if (tid == 0) L.bad = 1;
        __syncthreads();
        return;
    }
    if (warp == 0) {
        // experts in contiguous chunks per lane: scan of pair and expert counts
        const int chunk = (E + 31) / 32, e0 = min(E, lane * chunk), e1 = min(E, e0 + chunk);
        int np = 0, nu = 0;
        for (int e = e0; e < e1; ++e) {
            np += cnt[e];
            nu += cnt[e] > 0;
        }
        int ip = np, iu = nu;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int a = __shfl_up_sync(0xffffffffu, ip, o), b = __shfl_up_sync(0xffffffffu, iu, o);
            if (lane >= o) {
                ip += a;
                iu += b;
            }
        }
        int at = ip - np, u = iu - nu;
        for (int e = e0; e < e1; ++e) {
            const int c = cnt[e];
            if (c > 0) {
                L.off[u] = (int16_t)at;
                L.slot[u] = (int16_t)emap[e];
                base[e] = at;
                ++u;
                at += c;
            }
        }
        if (lane == 31) {
            L.nu = iu;
            L.off[iu] = (int16_t)P;
        }
        __syncwarp();
        // placement, 32 pairs at a time in ascending order
        for (int c0 = 0; c0 < P; c0 += 32) {
            const int p = c0 + lane;
            const int e = p < P ? ids[p] : -1 - lane;
            const unsigned peers = __match_any_sync(0xffffffffu, e);
            const int rank = __popc(peers & ((1u << lane) - 1u));
            if (p < P) L.pairs[base[e] + rank] = p;
            __syncwarp();
            if (p < P && rank == 0) base[e] += __popc(peers);
            __syncwarp();
        }
    }
    __syncthreads();
}

__global__ void __launch_bounds__(kThreads, 1)
    batch_moe_kernel(const __grid_constant__ CUtensorMap map_w13, const __grid_constant__ CUtensorMap map_w2,
                     const __grid_constant__ CUtensorMap map_x, const __grid_constant__ CUtensorMap map_act,
                     const Args g) {
    extern __shared__ unsigned char smem_raw[];
    __shared__ Ring R;
    __shared__ Lists L;
    unsigned char *stages = align1024(smem_raw);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int H = g.H, I = g.I;
    pdl_wait();
    pdl_launch_dependents();
    if (threadIdx.x == 0) trace_at(g.trace, kTrEntry);

    // the next launch's counters
    {
        const int gtid = blockIdx.x * blockDim.x + threadIdx.x, gstride = gridDim.x * blockDim.x;
        for (int i = gtid; i < kBatchReadyWords; i += gstride) g.ready_next[i] = 0;
        const int ndone = batch_done_words(g.H);
        for (int i = gtid; i < ndone; i += gstride) g.done_next[i] = 0;
    }

    // ---- the expert lists ----------------------------------------------------------
    const int32_t *pairs;
    if (g.route) {
        if (threadIdx.x == 0) L.bad = 0;
        __syncthreads();
        route_pairs(g, L, stages);
        if (L.bad) {
            if (blockIdx.x == 0 && threadIdx.x == 0) {
                *reinterpret_cast<volatile int32_t *>(g.dev_status) = WISP_ERR_BAD_EXPERT;
                if (g.status) *reinterpret_cast<volatile int *>(g.status) = WISP_ERR_BAD_EXPERT;
            }
            return;
        }
        pairs = L.pairs;
    } else {
        const int nu = min(gemm::group_experts(g.nu_dev, g.pager_status), kMaxPairs);
        for (int i = threadIdx.x; i <= nu; i += blockDim.x) L.off[i] = (int16_t)g.u_off[i];
        for (int i = threadIdx.x; i < nu; i += blockDim.x) L.slot[i] = (int16_t)g.u_slot[i];
        if (threadIdx.x == 0) L.nu = nu;
        pairs = g.u_pairs;
        __syncthreads();
    }
    if (warp == 0) {
        // token blocks per expert: prefix over experts in contiguous chunks per lane
        const int nu = L.nu, chunk = (nu + 31) / 32, e0 = min(nu, lane * chunk), e1 = min(nu, e0 + chunk);
        int nb = 0;
        for (int e = e0; e < e1; ++e) nb += (L.off[e + 1] - L.off[e] + kTN - 1) / kTN;
        int inc = nb;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int v = __shfl_up_sync(0xffffffffu, inc, o);
            if (lane >= o) inc += v;
        }
        int acc = inc - nb;
        for (int e = e0; e < e1; ++e) {
            L.first[e] = (int16_t)acc;
            acc += (L.off[e + 1] - L.off[e] + kTN - 1) / kTN;
        }
        if (lane == 31) {
            L.first[nu] = (int16_t)inc;
            L.nblocks = inc;
        }
    }
    __syncthreads();
    for (int b = threadIdx.x; b < L.nblocks; b += blockDim.x) {
        int u, q0, rows;
        block_of(L, b, u, q0, rows);
        L.rows[b] = (int16_t)rows;
    }
    __syncthreads();
    for (int b = threadIdx.x; b < L.nblocks; b += blockDim.x) {
        if (g.u_gen) {
            // experts still paging in: the pager's list order (resident experts
            // first, then the misses in page-in order), so tiles meet their
            // slots in the order the copies land
            L.order[b] = (int16_t)b;
            continue;
        }
        const int rb = L.rows[b];
        int rank = 0;
        for (int c = 0; c < L.nblocks; ++c) {
            const int rc = L.rows[c];
            rank += (rc > rb) || (rc == rb && c < b);
        }
        L.order[rank] = (int16_t)b;
    }
    if (threadIdx.x == 0) {
        R.abort = 0;
        R.issued = R.consumed = 0;
        if (g.route && blockIdx.x == 0) {
            // the pager's resident-mode bookkeeping: the forward, one group, its experts
            if (g.count_forward) g.hdr[1] += 1;
            g.hdr[5] += 1;
            g.hdr[6] += L.nu;
            *reinterpret_cast<volatile int32_t *>(g.dev_status) = WISP_OK;
        }
    }
    __syncthreads();
    if (threadIdx.x == 0) trace_at(g.trace, kTrLists);
    const int cj = I / kWM, ch = H / kDownRows;
    const int ngu = L.nblocks * cj;
    const int ntiles = ngu + L.nblocks * ch;
    if (g.route) {
        // this CTA's share of X_perm: rows blockIdx.x, + gridDim.x, ... (read back
        // by TMA in every CTA), then count the CTA in
        const int H8 = H / 8, P = g.T * g.K;
        for (int q = blockIdx.x; q < P; q += gridDim.x) {
            const uint4 *src = g.x + (size_t)(L.pairs[q] / g.K) * H8;
            uint4 *dst = g.x_perm + (size_t)q * H8;
            for (int c = threadIdx.x; c < H8; c += blockDim.x) dst[c] = src[c];
        }
        fence_proxy_async_global();
        __syncthreads();
        if (threadIdx.x == 0) red_release_gpu_add(g.ready + kGatheredWord, 1u);
    }
    if ((int)blockIdx.x >= ntiles) return;
    __syncthreads();  // the ring is no longer scratch

    if (threadIdx.x == 0) {
        for (int s = 0; s < kStages; ++s) {
            mbar_init(&R.full[s], 1);
            mbar_init(&R.empty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&R.acc_full[b], 1);
            mbar_init(&R.acc_empty[b], kEpiThreads);
        }
        mbar_init(&R.mma_done, 1);
        for (int k = 0; k < kTileRing; ++k) {
            mbar_init(&R.tile_full[k], 1);
            mbar_init(&R.tile_empty[k], 1 + kEpiWarps);
        }
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    }
    if (warp == 0) tmem_alloc(&R.tmem_base, kTmemCols);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (threadIdx.x == 0) trace_at(g.trace, kTrRoles);
    volatile int *abort = &R.abort;
    const uint32_t need = (uint32_t)(kEpiWarps * cj);

    if (warp == 0) {
        // ---- producer --------------------------------------------------------------
        if (lane == 0) {
            const uint64_t once = policy_evict_first();  // each weight tile is read once
            int kstep = 0;
            bool gathered = false;
            for (int i = 0;; ++i) {
                const int ts = i % kTileRing;
                if (i >= kTileRing &&
                    !mbar_wait(&R.tile_empty[ts], ((i / kTileRing) - 1) & 1, g.wait_ns, abort)) {
                    give_up(R, g);
                    break;
                }
                int t = (int)atomicAdd(g.ready + kSchedWord, 1u);
                if (t >= ntiles) t = -1;
                R.tile[ts] = t;
                mbar_arrive(&R.tile_full[ts]);
                if (t < 0) break;
                const Tile tl = tile_at(L, t, ngu, cj, ch);
                int u, q0, rows;
                block_of(L, tl.b, u, q0, rows);
                const int slot = L.slot[u];
                const CUtensorMap *mw, *mt;
                int a0, a1, kbc, kb0 = 0;
                if (!tl.down) {
                    mw = &map_w13;
                    mt = &map_x;
                    a0 = slot * 2 * I + tl.col * kWM;
                    a1 = a0 + I;
                    kbc = H / kBK;
                    if (g.u_gen && !wait_slot(g, u, slot, abort)) {
                        give_up(R, g);
                        break;
                    }
                    if (g.route && !gathered) {
                        // the weight boxes of the ring's unused stages go out now and
                        // stream while the other CTAs finish gathering the token rows;
                        // the token boxes follow the wait (issued even when the wait
                        // gives up, so every stage's transaction completes)
                        const int pre = max(0, min(kbc, kStages - kstep));
                        for (int q = 0; q < pre; ++q) {
                            const int s = kstep + q;
                            unsigned char *st = stages + s * kStageBytes;
                            mbar_expect_tx(&R.full[s], kStageBytes);
                            tma_load_2d_hint(st, mw, q * kBK, a0, &R.full[s], once);
                            tma_load_2d_hint(st + kWBoxBytes, mw, q * kBK, a1, &R.full[s], once);
                        }
                        if (pre > 0) trace_at(g.trace, kTrFirstLoad);
                        const bool ok = wait_ready(g, kGatheredWord, gridDim.x, abort);
                        for (int q = 0; q < pre; ++q) {
                            const int s = kstep + q;
                            tma_load_2d(stages + s * kStageBytes + 2 * kWBoxBytes, mt, q * kBK, q0, &R.full[s]);
                        }
                        kstep += pre;
                        kb0 = pre;
                        R.issued = kstep;
                        gathered = true;
                        if (!ok) {
                            give_up(R, g);
                            break;
                        }
                    }
                } else {
                    mw = &map_w2;
                    mt = &map_act;
                    a0 = slot * H + tl.col * kDownRows;
                    a1 = a0 + kWM;
                    kbc = I / kBK;
                    if (!wait_ready(g, tl.b, need, abort)) {
                        give_up(R, g);
                        break;
                    }
                }
                bool ok = true;
                for (int kb = kb0; kb < kbc; ++kb, ++kstep) {
                    const int s = kstep % kStages;
                    if (kstep >= kStages &&
                        !mbar_wait(&R.empty[s], ((kstep / kStages) - 1) & 1, g.wait_ns, abort)) {
                        ok = false;
                        break;
                    }
                    unsigned char *st = stages + s * kStageBytes;
                    mbar_expect_tx(&R.full[s], kStageBytes);
                    tma_load_2d_hint(st, mw, kb * kBK, a0, &R.full[s], once);
                    tma_load_2d_hint(st + kWBoxBytes, mw, kb * kBK, a1, &R.full[s], once);
                    tma_load_2d(st + 2 * kWBoxBytes, mt, kb * kBK, q0, &R.full[s]);
                    if (kstep == 0) trace_at(g.trace, kTrFirstLoad);
                    R.issued = kstep + 1;
                }
                if (!ok) {
                    give_up(R, g);
                    break;
                }
            }
            trace_at(g.trace, kTrLastLoad);
        }
    } else if (warp == 1) {
        // ---- MMA issuer -------------------------------------------------------------
        if (lane == 0) {
            const uint32_t idesc = gemm::idesc_bf16_f32(kWM, kTN);
            int kstep = 0;
            for (int i = 0;; ++i) {
                const int t = next_tile(R, i, g, true);
                if (t < 0) break;
                const int kbc = (t < ngu ? H : I) / kBK;
                const int b = i & 1;
                if (i >= 2 && !mbar_wait(&R.acc_empty[b], ((i / 2) - 1) & 1, g.wait_ns, abort)) {
                    give_up(R, g);
                    break;
                }
                tc_fence_after();
                const uint32_t acc = R.tmem_base + b * kAccCols;
                bool ok = true;
                for (int kb = 0; kb < kbc; ++kb, ++kstep) {
                    const int s = kstep % kStages;
                    if (!mbar_wait(&R.full[s], (kstep / kStages) & 1, g.wait_ns, abort)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t w0 = s_addr(stages + s * kStageBytes), w1 = w0 + kWBoxBytes,
                                   tk = w0 + 2 * kWBoxBytes;
#pragma unroll
                    for (int kk = 0; kk < kBK / 16; ++kk) {  // 16 bf16 = 32 bytes further along K
                        const uint64_t bdesc = smem_desc_k_sw128(tk + kk * 32);
                        const uint32_t accumulate = (kb | kk) != 0;
                        umma_f16(acc, smem_desc_k_sw128(w0 + kk * 32), bdesc, idesc, accumulate);
                        umma_f16(acc + kTN, smem_desc_k_sw128(w1 + kk * 32), bdesc, idesc, accumulate);
                    }
                    umma_commit(&R.empty[s]);
                    R.consumed = kstep + 1;
                }
                if (!ok) {
                    give_up(R, g);
                    break;
                }
                umma_commit(&R.acc_full[b]);
            }
            umma_commit(&R.mma_done);  // every MMA issued (also after an abort)
            trace_at(g.trace, kTrLastMma);
        }
    } else {
        // ---- epilogue (warps 2..5) ----------------------------------------------------
        const int quarter = warp & 3, r = quarter * 32 + lane;
        for (int i = 0;; ++i) {
            int t = next_tile(R, i, g, false);
            t = __shfl_sync(0xffffffffu, t, 0);
            __syncwarp();
            if (lane == 0 && t >= 0) mbar_arrive(&R.tile_empty[i % kTileRing]);
            if (t < 0) break;
            const bool ok = mbar_wait(&R.acc_full[i & 1], (i / 2) & 1, g.wait_ns, abort) && !*abort;
            if (!__all_sync(0xffffffffu, ok)) break;  // uniform: the TMEM loads are .sync.aligned
            tc_fence_after();
            const Tile tl = tile_at(L, t, ngu, cj, ch);
            int u, q0, rows;
            block_of(L, tl.b, u, q0, rows);
            const uint32_t tbase = R.tmem_base + (i & 1) * kAccCols + ((uint32_t)(quarter * 32) << 16);
            uint32_t d0[kTN], d1[kTN];
            tmem_ld32(tbase, d0);
            tmem_ld32(tbase + kTN, d1);
            tc_fence_before();
            mbar_arrive(&R.acc_empty[i & 1]);  // the values are in registers
            if (!tl.down) {
                __nv_bfloat16 *dst = g.act_perm + (size_t)q0 * I + tl.col * kWM + r;
#pragma unroll
                for (int n = 0; n < kTN; ++n) {
                    if (n < rows) {
                        const float gv = round_bf16(__uint_as_float(d0[n]));
                        const float uv = round_bf16(__uint_as_float(d1[n]));
                        dst[(size_t)n * I] = act_value(silu_stored(gv) * uv);
                    }
                }
                fence_proxy_async_global();
                __syncwarp();
                if (lane == 0) red_release_gpu_add(g.ready + tl.b, 1u);
            } else {
                const int h = tl.col * kDownRows + r;
#pragma unroll
                for (int n = 0; n < kTN; ++n) {
                    if (n < rows) {
                        const int p = pairs[q0 + n];
                        const float wp = g.topk_w[p];
                        __nv_bfloat16 *dst = g.y + (size_t)p * H + h;
                        dst[0] = __float2bfloat16_rn(__uint_as_float(d0[n]) * wp);
                        dst[kWM] = __float2bfloat16_rn(__uint_as_float(d1[n]) * wp);
                    }
                }
                combine_rows(g, pairs, q0, rows, tl.col, quarter, lane, h);
            }
        }
        if (warp == 2 && lane == 0) trace_at(g.trace, kTrEpiDone);
    }

    // ---- teardown ----------------------------------------------------------------------
    tc_fence_before();
    __syncthreads();
    if (R.abort && threadIdx.x == 0) {
        // wait, bounded, for the copies issued but not consumed and the MMAs issued
        volatile int no_abort = 0;
        for (int k = R.consumed; k < R.issued; ++k)
            mbar_wait(&R.full[k % kStages], (k / kStages) & 1, g.wait_ns, &no_abort);
        mbar_wait(&R.mma_done, 0, g.wait_ns, &no_abort);
    }
    __syncthreads();
    tc_fence_after();
    if (warp == 0) tmem_dealloc(R.tmem_base, kTmemCols);
    if (threadIdx.x == 0) trace_at(g.trace, kTrExit);
}

// Shared launch of the persistent kernel (cooperative: at most one CTA per
// SM, all resident -- the down tiles wait for gate-up tiles of other CTAs).
int launch_kernel(const PrefillGroup &p, const Args &a, long nu_bound, cudaStream_t stream) {
    static bool attr_set[64] = {};
    int dev = 0;
    WISP_CUDA_TRY(cudaGetDevice(&dev));
    if (dev < 0 || dev >= 64) return WISP_ERR_INVALID;
    if (!attr_set[dev]) {
        WISP_CUDA_TRY(cudaFuncSetAttribute(batch_moe_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes));
        attr_set[dev] = true;
    }
    CUtensorMap mw13, mw2, mx, mact;
    int rc = gemm::make_map(&mw13, p.w13, (uint64_t)p.slots * 2 * p.I, (uint64_t)p.H, kWM);
    if (!rc) rc = gemm::make_map(&mw2, p.w2, (uint64_t)p.slots * p.H, (uint64_t)p.I, kWM);
    if (!rc) rc = gemm::make_map(&mx, p.x_perm, (uint64_t)p.perm_rows, (uint64_t)p.H, kTN);
    if (!rc) rc = gemm::make_map(&mact, p.act_perm, (uint64_t)p.perm_rows, (uint64_t)p.I, kTN);
    if (rc) return rc;
    int sms = 0;
    WISP_CUDA_TRY(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
    const long blocks = std::min<long>(nu_bound, p.npairs) + (p.npairs + kTN - 1) / kTN;
    const long tiles = blocks * (p.I / kWM + p.H / kDownRows);
    return launch_persistent(batch_moe_kernel, dim3((unsigned)std::max<long>(1, std::min<long>(tiles, sms))),
                             dim3(kThreads), (size_t)kSmemBytes, stream, mw13, mw2, mx, mact, a);
}

int check_group(const PrefillGroup &p, const BatchCounters &c) {
    if (!prefill_shapes_supported(p.H, p.I))
        return set_error("wisp: tensor-core path needs hidden % 256 == 0 and inter % 128 == 0"), WISP_ERR_UNSUPPORTED;
    if (p.npairs > kMaxPairs)
        return set_error("wisp: weight-stationary path takes at most 512 pairs per call"), WISP_ERR_INVALID;
    if (!c.ready || !c.ready_next || !c.done || !c.done_next)
        return set_error("wisp: batch path without its counters"), WISP_ERR_INVALID;
    return WISP_OK;
}

Args common_args(const PrefillGroup &p, const BatchCounters &c) {
    Args a{};
    a.H = p.H;
    a.I = p.I;
    a.Kc = p.K;
    a.t0 = p.t0;
    a.topk_w = p.topk_w;
    a.act_perm = p.act_perm;
    a.y = p.y;
    a.out = p.out;
    a.ready = c.ready;
    a.ready_next = c.ready_next;
    a.done = c.done;
    a.done_next = c.done_next;
    a.status = p.status;
    a.wait_ns = p.wait_ns;
    a.trace = p.trace;
    return a;
}

}  // namespace
}  // namespace batch

int launch_batch_group(const PrefillGroup &p, const BatchCounters &c, cudaStream_t stream) {
    using namespace batch;
    int rc = check_group(p, c);
    if (rc || p.npairs <= 0 || p.nu <= 0) return rc;
    Args a = common_args(p, c);
    a.u_off = p.u_off;
    a.u_pairs = p.u_pairs;
    a.u_slot = p.u_slot;
    a.nu_dev = p.nu_dev;
    a.pager_status = p.pager_status;
    a.u_gen = p.u_gen;
    a.slot_ready = p.slot_ready;
    rc = gemm::launch_gather(p, stream);
    if (!rc) rc = launch_kernel(p, a, p.nu, stream);
    return rc;
}

int launch_batch_resident(const PrefillGroup &p, const BatchRoute &r, const BatchCounters &c, cudaStream_t stream) {
    using namespace batch;
    int rc = check_group(p, c);
    if (rc || p.npairs <= 0) return rc;
    if (r.E < 1 || r.E > kMaxRouteExperts)
        return set_error("wisp: in-kernel routing takes at most 1024 experts"), WISP_ERR_INVALID;
    Args a = common_args(p, c);
    a.route = 1;
    a.ids = r.ids;
    a.ids64 = r.ids64;
    a.T = p.t1 - p.t0;
    a.K = p.K;
    a.E = r.E;
    a.count_forward = r.count_forward;
    a.emap = r.emap;
    a.x = reinterpret_cast<const uint4 *>(p.x);
    a.x_perm = reinterpret_cast<uint4 *>(p.x_perm);
    a.hdr = r.hdr;
    a.dev_status = r.dev_status;
    return launch_kernel(p, a, std::min(r.E, p.npairs), stream);
}

}  // namespace wisp
