// Expert-parallel token exchange over peer memory (NVLink / NVSwitch).
//
// Rank r of `world` owns experts [r * experts_per_rank, (r + 1) *
// experts_per_rank).  Each rank allocates one symmetric region (the same
// layout on every rank) and maps every peer's region through CUDA IPC, so a
// kernel on one GPU stores straight into another GPU's HBM:
//
//   inbox      [world] {count, source pairs, epoch}: written by each source
//   back_flag  [world] {epoch}: written by each owner when this rank's rows
//              are back
//   recs       [world][max_pairs] {local expert id, weight bits, source pair, 0}
//   recv       [world][max_pairs][H] bf16: source s's rows for this owner
//   back       [max_pairs][H] bf16: this rank's weighted rows, by pair t*k+j
//
// One forward of one layer, per rank (every rank calls the same sequence;
// each call bumps the group's epoch, so no flag is ever reset):
//
//   ep_dispatch_kernel  every CTA routes the call's (token, k) pairs (owner,
//                       stable position within the owner: pairs keep their
//                       (t, k) order), warps store x rows and records into
//                       the owners' recv segments; the last CTA to finish
//                       publishes {count, pairs} and then the epoch in every
//                       owner's inbox (release at system scope);
//   ep_receive_kernel   waits (bounded) for every source's epoch, compacts
//                       the received rows for the owner's local paged layer
//                       and reports the counts to the host (the local forward
//                       needs its row count).  Rows keep their run of sources
//                       (consecutive sources of one compute class, in rank
//                       order) and are ordered within it by local expert,
//                       stably, so the pager pages each expert of a run once;
//   (the owner's layer forward on the compacted rows, top_k 1)
//   ep_return_kernel    stores each weighted row into its source's back
//                       buffer at the source's pair index; the last CTA
//                       raises this owner's flag in every source's back_flag;
//   ep_combine_kernel   waits (bounded) for every owner's flag and writes
//                       out[t] = routing-order sum of back[t*k + j]
//                       (combine_add: bf16 partial sums up to top-4, fp32
//                       above), stored bf16 -- the one-GPU combine.
//
// Ordering argument (one buffer set serves every layer): a source's next
// dispatch comes after its combine, which waited for every owner's return,
// which each owner issues after its receive finished reading the recv
// segments; an owner writes a source's back rows only after that source's
// dispatch of the same epoch, which followed the source's previous combine.
//
// No collective library is on the data path; every store to a peer is a
// plain generic store from these kernels (no TMA, no library kernel touches
// peer memory).
#include <mutex>
#include <string>
#include <vector>

#include "common.cuh"

namespace {

constexpr int kMaxRanks = 64;
constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr int kMaxPairsLimit = 1 << 15;  // positions and pair indices packed in 16 bits
constexpr int kMaxRecvRows = 48 * 1024;  // rows one owner can receive (the receive kernel's ordering in shared memory)

size_t align256(size_t v) { return (v + 255) & ~size_t(255); }

struct Layout {
    size_t inbox, back_flag, recs, recv, back, total;
};

Layout make_layout(int world, int max_pairs, int H) {
    Layout l{};
    size_t o = 0;
    l.inbox = o;
    o = align256(o + 16 * (size_t)world);
    l.back_flag = o;
    o = align256(o + 16 * (size_t)world);
    l.recs = o;
    o = align256(o + 16 * (size_t)world * max_pairs);
    l.recv = o;
    o = align256(o + 2 * (size_t)world * max_pairs * H);
    l.back = o;
    o = align256(o + 2 * (size_t)max_pairs * H);
    l.total = o;
    return l;
}

}  // namespace

struct wisp_ep_group {
    int rank = 0, world = 1, dev = 0, max_pairs = 0, H = 0;
    Layout lay{};
    char *base = nullptr;                 // this rank's symmetric region
    std::vector<char *> peer;             // every rank's region as this device sees it
    std::vector<bool> opened;             // peer[i] came from cudaIpcOpenMemHandle
    char **d_peer = nullptr;              // device copy of peer[]
    unsigned int *d_counter = nullptr;    // [2] last-CTA counters (dispatch, return)
    int *d_status = nullptr;              // sticky device status of the group's kernels
    // owner side: the compacted received rows for the local layer
    __nv_bfloat16 *x_recv = nullptr, *y_recv = nullptr;
    int32_t *ids_recv = nullptr, *map_recv = nullptr;
    float *w_recv = nullptr;
    int32_t *h_info = nullptr, *d_info = nullptr;  // mapped: status, R, counts[world], pairs[world]
    cudaEvent_t ev = nullptr;
    int epoch = 0;
    int last_R = 0;
    int e_local = 1;                      // experts per rank of the last dispatch
    size_t recv_smem = 48 * 1024;         // dynamic shared memory the receive kernel may use
    long long wait_ns = 10LL * 1000 * 1000 * 1000;
    std::mutex mu;
};

namespace wisp {
namespace ep {
namespace {

struct alignas(16) Inbox {
    int count, src_pairs, epoch, pad;
};

__device__ __forceinline__ void st_release_sys(int *p, int v) {
    asm volatile("st.release.sys.global.b32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ int ld_acquire_sys(const int *p) {
    int v;
    asm volatile("ld.acquire.sys.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// Bounded wait (thread 0 of a CTA) until words[i * stride_words].epoch ==
// epoch for every i < n; false when the limit ran out.
__device__ bool wait_epochs(const int *first_epoch_word, int stride_words, int n, int epoch, long long wait_ns) {
    const unsigned long long t0 = globaltimer_ns();
    for (int i = 0; i < n; ++i) {
        const int *w = first_epoch_word + (size_t)i * stride_words;
        while (ld_acquire_sys(w) != epoch) {
            if ((long long)(globaltimer_ns() - t0) > wait_ns) return false;
            __nanosleep(64);
        }
    }
    return true;
}

struct DispatchArgs {
    const uint4 *x;
    const void *ids;
    int ids64;
    const float *w;
    int P, K, H8, e_local, world, rank, max_pairs, epoch;
    char *const *peer;
    size_t off_inbox, off_recs, off_recv;
    unsigned int *counter;
};

// Every CTA routes all pairs (same result everywhere), then copies its share.
__global__ void __launch_bounds__(kThreads) ep_dispatch_kernel(const DispatchArgs a) {
    extern __shared__ int s_route[];  // [P]: (owner << 16) | position within the owner's segment
    __shared__ int s_cnt[kMaxRanks], s_base[kMaxRanks], s_wcnt[kWarps][kMaxRanks];
    __shared__ int s_last;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const long long E = (long long)a.e_local * a.world;
    for (int d = tid; d < a.world; d += kThreads) s_cnt[d] = 0;
    __syncthreads();
    int bad = 0;
    for (int p = tid; p < a.P; p += kThreads) {
        const long long e = load_id64(a.ids, a.ids64, p);
        if (e < 0 || e >= E)
            bad = 1;
        else
            atomicAdd(&s_cnt[(int)(e / a.e_local)], 1);
    }
    bad = __syncthreads_or(bad);
    if (!bad) {
        // each (source, owner) segment starts at row 0 of the owner's receive buffer
        for (int d = tid; d < a.world; d += kThreads) s_base[d] = 0;
        __syncthreads();
        const unsigned lt = (1u << lane) - 1u;
        for (int c0 = 0; c0 < a.P; c0 += kThreads) {
            for (int i = tid; i < kWarps * kMaxRanks; i += kThreads) (&s_wcnt[0][0])[i] = 0;
            __syncthreads();
            const int p = c0 + tid;
            int d = kMaxRanks + lane;  // never matches a real owner
            if (p < a.P) d = (int)(load_id64(a.ids, a.ids64, p) / a.e_local);
            const unsigned same = __match_any_sync(0xffffffffu, d);
            const int r = __popc(same & lt);
            if (p < a.P && r == 0) s_wcnt[warp][d] = __popc(same);
            __syncthreads();
            if (p < a.P) {
                int off = s_base[d] + r;
                for (int w = 0; w < warp; ++w) off += s_wcnt[w][d];
                s_route[p] = (d << 16) | off;
            }
            __syncthreads();
            for (int dd = tid; dd < a.world; dd += kThreads) {
                int tot = 0;
                for (int w = 0; w < kWarps; ++w) tot += s_wcnt[w][dd];
                s_base[dd] += tot;
            }
            __syncthreads();
        }
        // rows and records into the owners' segments (a warp per pair)
        for (int p = blockIdx.x * kWarps + warp; p < a.P; p += gridDim.x * kWarps) {
            const int v = s_route[p], d = v >> 16, j = v & 0xffff;
            char *owner = a.peer[d];
            const size_t row = (size_t)a.rank * a.max_pairs + j;
            uint4 *dst = reinterpret_cast<uint4 *>(owner + a.off_recv) + row * a.H8;
            const uint4 *src = a.x + (size_t)(p / a.K) * a.H8;
            for (int c = lane; c < a.H8; c += 32) dst[c] = src[c];
            if (lane == 0) {
                const long long e = load_id64(a.ids, a.ids64, p);
                uint4 rec;
                rec.x = (unsigned)(e - (long long)d * a.e_local);
                rec.y = __float_as_uint(a.w[p]);
                rec.z = (unsigned)p;
                rec.w = 0u;
                reinterpret_cast<uint4 *>(owner + a.off_recs)[row] = rec;
            }
        }
    }
    __threadfence_system();  // this thread's stores to peers, before the count-in
    __syncthreads();
    if (tid == 0) s_last = atomicAdd(a.counter, 1u) == gridDim.x - 1;
    __syncthreads();
    if (!s_last) return;
    __threadfence_system();
    for (int d = tid; d < a.world; d += kThreads) {
        Inbox *ib = reinterpret_cast<Inbox *>(a.peer[d] + a.off_inbox) + a.rank;
        ib->count = bad ? -1 : s_cnt[d];  // -1: this source routed an id out of range
        ib->src_pairs = a.P;
    }
    __threadfence_system();
    __syncthreads();
    for (int d = tid; d < a.world; d += kThreads)
        st_release_sys(&(reinterpret_cast<Inbox *>(a.peer[d] + a.off_inbox) + a.rank)->epoch, a.epoch);
    if (tid == 0) *a.counter = 0u;
}

struct ReceiveArgs {
    const char *base;
    size_t off_inbox, off_recs, off_recv;
    int world, max_pairs, H8, epoch, e_local;
    int class_min_pairs;  // > 0: sources of >= this many pairs form their own runs
    long long wait_ns;
    uint4 *x_recv;
    int32_t *ids_recv, *map_recv;
    float *w_recv;
    int32_t *info;   // mapped host: [0] status [1] R [2..) counts [2 + world ..) source pairs
};

// Row i of the received rows in (source, pair) order: its source.
__device__ __forceinline__ int source_of(const int *pre, int world, int i) {
    int s = 0;
    while (s + 1 < world && pre[s + 1] <= i) ++s;
    return s;
}

// Every CTA builds the same permutation: the rows of each run of sources
// (consecutive sources with rows, of one class) stay in that run's range and
// are ordered there by local expert, stably ((source, pair) order within an
// expert), so the owner's pager pages each expert of a run once.
__global__ void __launch_bounds__(kThreads) ep_receive_kernel(const ReceiveArgs a) {
    extern __shared__ int s_dyn[];  // [rows] destination of each row, then [e_local] expert counters
    __shared__ int s_cnt[kMaxRanks], s_pre[kMaxRanks + 1], s_run_start[kMaxRanks + 1];
    __shared__ int s_ok, s_bad, s_runs;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const Inbox *inbox = reinterpret_cast<const Inbox *>(a.base + a.off_inbox);
    if (tid == 0) s_ok = wait_epochs(&inbox[0].epoch, 4, a.world, a.epoch, a.wait_ns);
    __syncthreads();
    if (!s_ok) {  // reported by wisp_ep_receive itself (not sticky)
        if (blockIdx.x == 0 && tid == 0) {
            a.info[0] = WISP_ERR_TIMEOUT;
            a.info[1] = 0;
        }
        return;
    }
    for (int s = tid; s < a.world; s += kThreads)
        s_cnt[s] = *reinterpret_cast<const volatile int *>(&inbox[s].count);
    __syncthreads();
    if (tid == 0) {
        int run = 0, bad = 0, runs = 0, cls_prev = -1;
        for (int s = 0; s < a.world; ++s) {
            s_pre[s] = run;
            bad |= s_cnt[s] < 0;
            const int c = s_cnt[s] < 0 ? 0 : s_cnt[s];
            if (c > 0) {
                const int pairs = *reinterpret_cast<const volatile int *>(&inbox[s].src_pairs);
                const int cls = a.class_min_pairs > 0 && pairs >= a.class_min_pairs;
                if (cls != cls_prev) s_run_start[runs++] = run;
                cls_prev = cls;
            }
            run += c;
        }
        s_pre[a.world] = bad ? 0 : run;
        s_run_start[runs] = run;
        s_runs = runs;
        s_bad = bad;
    }
    __syncthreads();
    const int R = s_pre[a.world];
    if (blockIdx.x == 0) {
        for (int s = tid; s < a.world; s += kThreads) {
            a.info[2 + s] = s_cnt[s];
            a.info[2 + a.world + s] = *reinterpret_cast<const volatile int *>(&inbox[s].src_pairs);
        }
        if (tid == 0) {
            a.info[1] = R;
            a.info[0] = s_bad ? WISP_ERR_BAD_EXPERT : WISP_OK;
        }
    }
    if (s_bad) return;
    const uint4 *recs = reinterpret_cast<const uint4 *>(a.base + a.off_recs);
    const uint4 *recv = reinterpret_cast<const uint4 *>(a.base + a.off_recv);
    int *dest = s_dyn;
    int *ecnt = s_dyn + (size_t)a.world * a.max_pairs;
    for (int ru = 0; ru < s_runs; ++ru) {
        const int r0 = s_run_start[ru], r1 = s_run_start[ru + 1];
        for (int e = tid; e < a.e_local; e += kThreads) ecnt[e] = 0;
        __syncthreads();
        for (int i = r0 + tid; i < r1; i += kThreads) {
            const int s = source_of(s_pre, a.world, i);
            const int e = (int)__ldcg(&recs[(size_t)s * a.max_pairs + (i - s_pre[s])].x);
            atomicAdd(&ecnt[min(max(e, 0), a.e_local - 1)], 1);
        }
        __syncthreads();
        if (tid == 0) {
            int run = r0;
            for (int e = 0; e < a.e_local; ++e) {
                const int c = ecnt[e];
                ecnt[e] = run;
                run += c;
            }
        }
        __syncthreads();
        if (warp == 0) {
            // stable placement, 32 rows at a time in (source, pair) order
            const unsigned lt = (1u << lane) - 1u;
            for (int c0 = r0; c0 < r1; c0 += 32) {
                const int i = c0 + lane;
                int e = a.e_local + lane;  // never matches a real expert
                if (i < r1) {
                    const int s = source_of(s_pre, a.world, i);
                    e = min(max((int)__ldcg(&recs[(size_t)s * a.max_pairs + (i - s_pre[s])].x), 0), a.e_local - 1);
                }
                const unsigned same = __match_any_sync(0xffffffffu, e);
                const int rk = __popc(same & lt);
                if (i < r1) dest[i] = ecnt[e] + rk;
                __syncwarp();
                if (i < r1 && rk == 0) ecnt[e] += __popc(same);
                __syncwarp();
            }
        }
        __syncthreads();
    }
    for (int i = blockIdx.x * kWarps + warp; i < R; i += gridDim.x * kWarps) {
        const int s = source_of(s_pre, a.world, i);
        const size_t row = (size_t)s * a.max_pairs + (i - s_pre[s]);
        const int d = dest[i];
        const uint4 *src = recv + row * a.H8;
        uint4 *dst = a.x_recv + (size_t)d * a.H8;
        for (int c = lane; c < a.H8; c += 32) dst[c] = __ldcg(src + c);
        if (lane == 0) {
            const uint4 rec = __ldcg(recs + row);
            a.ids_recv[d] = (int)rec.x;
            a.w_recv[d] = __uint_as_float(rec.y);
            a.map_recv[d] = (s << 16) | (int)rec.z;
        }
    }
}

struct ReturnArgs {
    const uint4 *y_recv;
    const int32_t *map_recv;
    int R, H8, world, rank, epoch;
    char *const *peer;
    size_t off_back, off_back_flag;
    unsigned int *counter;
};

__global__ void __launch_bounds__(kThreads) ep_return_kernel(const ReturnArgs a) {
    __shared__ int s_last;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    for (int i = blockIdx.x * kWarps + warp; i < a.R; i += gridDim.x * kWarps) {
        const int m = a.map_recv[i], s = m >> 16, pair = m & 0xffff;
        uint4 *dst = reinterpret_cast<uint4 *>(a.peer[s] + a.off_back) + (size_t)pair * a.H8;
        const uint4 *src = a.y_recv + (size_t)i * a.H8;
        for (int c = lane; c < a.H8; c += 32) dst[c] = src[c];
    }
    __threadfence_system();
    __syncthreads();
    if (tid == 0) s_last = atomicAdd(a.counter, 1u) == gridDim.x - 1;
    __syncthreads();
    if (!s_last) return;
    __threadfence_system();
    for (int s = tid; s < a.world; s += kThreads)
        st_release_sys(reinterpret_cast<int *>(a.peer[s] + a.off_back_flag) + 4 * a.rank, a.epoch);
    if (tid == 0) *a.counter = 0u;
}

struct CombineArgs {
    const char *base;
    size_t off_back, off_back_flag;
    int world, T, K, H8, epoch;
    long long wait_ns;
    uint4 *out;
    int *status;
};

__global__ void __launch_bounds__(kThreads) ep_combine_kernel(const CombineArgs a) {
    __shared__ int s_ok;
    if (threadIdx.x == 0)
        s_ok = wait_epochs(reinterpret_cast<const int *>(a.base + a.off_back_flag), 4, a.world, a.epoch,
                           a.wait_ns);
    __syncthreads();
    if (!s_ok) {
        if (threadIdx.x == 0) *a.status = WISP_ERR_TIMEOUT;
        return;
    }
    const uint4 *back = reinterpret_cast<const uint4 *>(a.base + a.off_back);
    const long n = (long)a.T * a.H8;
    for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long)gridDim.x * blockDim.x) {
        const int t = (int)(i / a.H8), c = (int)(i - (long)t * a.H8);
        float acc[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[j] = 0.f;
        for (int k = 0; k < a.K; ++k) {
            const uint4 v = __ldcg(back + ((size_t)t * a.K + k) * a.H8 + c);
            const uint32_t wv[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                acc[2 * j] = combine_add(acc[2 * j], bf16lo(wv[j]), a.K);
                acc[2 * j + 1] = combine_add(acc[2 * j + 1], bf16hi(wv[j]), a.K);
            }
        }
        uint32_t o[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const uint32_t lo = __bfloat16_as_ushort(__float2bfloat16_rn(acc[2 * j]));
            const uint32_t hi = __bfloat16_as_ushort(__float2bfloat16_rn(acc[2 * j + 1]));
            o[j] = lo | (hi << 16);
        }
        a.out[i] = make_uint4(o[0], o[1], o[2], o[3]);
    }
}

int fail(int code, const std::string &msg) {
    set_error(msg);
    return code;
}

struct Guard {
    int prev = -1;
    explicit Guard(int dev) {
        if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
        if (prev != dev) cudaSetDevice(dev);
    }
    ~Guard() {
        if (prev >= 0) cudaSetDevice(prev);
    }
};

int grid_for(long work_warps, int dev) {
    int sms = 148;
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) sms = 148;
    const long g = (work_warps + kWarps - 1) / kWarps;
    return (int)std::max<long>(1, std::min<long>(g, 2L * sms));
}

}  // namespace
}  // namespace ep
}  // namespace wisp

using namespace wisp;
using namespace wisp::ep;

extern "C" {

int wisp_ep_group_create(int32_t rank, int32_t world, int32_t device, int32_t max_pairs, int32_t hidden,
                         wisp_ep_group **out) {
    if (!out) return fail(WISP_ERR_INVALID, "wisp_ep_group_create: out is NULL");
    *out = nullptr;
    if (world < 1 || world > kMaxRanks || rank < 0 || rank >= world)
        return fail(WISP_ERR_INVALID, "wisp_ep_group_create: need 0 <= rank < world <= 64");
    if (max_pairs < 1 || max_pairs > kMaxPairsLimit)
        return fail(WISP_ERR_INVALID, "wisp_ep_group_create: max_pairs must be in [1, 32768]");
    if (hidden < 8 || hidden % 8) return fail(WISP_ERR_INVALID, "wisp_ep_group_create: hidden a multiple of 8");
    if ((long)world * max_pairs > kMaxRecvRows)
        return fail(WISP_ERR_INVALID, "wisp_ep_group_create: world * max_pairs must be at most " +
                                          std::to_string(kMaxRecvRows));
    if (device < 0) return fail(WISP_ERR_INVALID, "wisp_ep_group_create: bad device");
    Guard guard(device);
    auto *g = new wisp_ep_group();
    g->rank = rank;
    g->world = world;
    g->dev = device;
    g->max_pairs = max_pairs;
    g->H = hidden;
    g->lay = make_layout(world, max_pairs, hidden);
    g->peer.assign(world, nullptr);
    g->opened.assign(world, false);
    const size_t nrecv = (size_t)world * max_pairs;
    auto bail = [&](const char *what) {
        wisp_ep_group_destroy(g);
        return fail(WISP_ERR_NOMEM, std::string("wisp_ep_group_create: ") + what);
    };
    if (cudaMalloc(&g->base, g->lay.total) != cudaSuccess) return bail("symmetric region");
    if (cudaMemset(g->base, 0, g->lay.total) != cudaSuccess) return bail("clearing the region");
    if (cudaMalloc(&g->d_peer, sizeof(char *) * world) != cudaSuccess ||
        cudaMalloc(&g->d_counter, sizeof(unsigned int) * 2) != cudaSuccess ||
        cudaMalloc(&g->d_status, sizeof(int)) != cudaSuccess ||
        cudaMalloc(&g->x_recv, sizeof(__nv_bfloat16) * nrecv * hidden) != cudaSuccess ||
        cudaMalloc(&g->y_recv, sizeof(__nv_bfloat16) * nrecv * hidden) != cudaSuccess ||
        cudaMalloc(&g->ids_recv, sizeof(int32_t) * nrecv) != cudaSuccess ||
        cudaMalloc(&g->map_recv, sizeof(int32_t) * nrecv) != cudaSuccess ||
        cudaMalloc(&g->w_recv, sizeof(float) * nrecv) != cudaSuccess)
        return bail("device buffers");
    if (cudaHostAlloc(&g->h_info, sizeof(int32_t) * (2 + 2 * world), cudaHostAllocMapped) != cudaSuccess ||
        cudaHostGetDevicePointer((void **)&g->d_info, g->h_info, 0) != cudaSuccess)
        return bail("mapped status words");
    if (cudaMemset(g->d_counter, 0, sizeof(unsigned int) * 2) != cudaSuccess ||
        cudaMemset(g->d_status, 0, sizeof(int)) != cudaSuccess ||
        cudaEventCreateWithFlags(&g->ev, cudaEventDisableTiming) != cudaSuccess ||
        cudaDeviceSynchronize() != cudaSuccess)
        return bail("initialisation");
    g->peer[rank] = g->base;
    *out = g;
    return WISP_OK;
}

int wisp_ep_group_ipc_handle(wisp_ep_group *g, void *handle_out) {
    if (!g || !handle_out) return fail(WISP_ERR_INVALID, "wisp_ep_group_ipc_handle: NULL argument");
    Guard guard(g->dev);
    cudaIpcMemHandle_t h;
    WISP_CUDA_TRY(cudaIpcGetMemHandle(&h, g->base));
    memcpy(handle_out, &h, sizeof(h));
    return WISP_OK;
}

int wisp_ep_group_connect(wisp_ep_group *g, const void *handles) {
    if (!g || !handles) return fail(WISP_ERR_INVALID, "wisp_ep_group_connect: NULL argument");
    Guard guard(g->dev);
    const char *hb = reinterpret_cast<const char *>(handles);
    for (int r = 0; r < g->world; ++r) {
        if (r == g->rank || g->peer[r]) continue;
        cudaIpcMemHandle_t h;
        memcpy(&h, hb + (size_t)r * sizeof(cudaIpcMemHandle_t), sizeof(h));
        void *p = nullptr;
        WISP_CUDA_TRY(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess));
        g->peer[r] = reinterpret_cast<char *>(p);
        g->opened[r] = true;
    }
    WISP_CUDA_TRY(cudaMemcpy(g->d_peer, g->peer.data(), sizeof(char *) * g->world, cudaMemcpyHostToDevice));
    return WISP_OK;
}

int wisp_ep_group_connect_local(wisp_ep_group *g, wisp_ep_group *const *groups) {
    if (!g || !groups) return fail(WISP_ERR_INVALID, "wisp_ep_group_connect_local: NULL argument");
    Guard guard(g->dev);
    for (int r = 0; r < g->world; ++r) {
        const wisp_ep_group *o = groups[r];
        if (!o || o->world != g->world || o->rank != r || o->max_pairs != g->max_pairs || o->H != g->H ||
            o->dev != g->dev)
            return fail(WISP_ERR_INVALID,
                        "wisp_ep_group_connect_local: groups[r] must be rank r of the same shape on this device");
        g->peer[r] = o->base;
    }
    WISP_CUDA_TRY(cudaMemcpy(g->d_peer, g->peer.data(), sizeof(char *) * g->world, cudaMemcpyHostToDevice));
    return WISP_OK;
}

int wisp_ep_group_destroy(wisp_ep_group *g) {
    if (!g) return WISP_OK;
    {
        Guard guard(g->dev);
        cudaDeviceSynchronize();
        for (int r = 0; r < g->world; ++r)
            if (g->opened[r] && g->peer[r]) cudaIpcCloseMemHandle(g->peer[r]);
        for (void *p : {(void *)g->base, (void *)g->d_peer, (void *)g->d_counter, (void *)g->d_status,
                        (void *)g->x_recv, (void *)g->y_recv, (void *)g->ids_recv, (void *)g->map_recv,
                        (void *)g->w_recv})
            if (p) cudaFree(p);
        if (g->h_info) cudaFreeHost(g->h_info);
        if (g->ev) cudaEventDestroy(g->ev);
    }
    delete g;
    return WISP_OK;
}

int wisp_ep_group_buffers(wisp_ep_group *g, void **x_recv, void **ids_recv, void **w_recv, void **y_recv) {
    if (!g) return fail(WISP_ERR_INVALID, "wisp_ep_group_buffers: NULL group");
    if (x_recv) *x_recv = g->x_recv;
    if (ids_recv) *ids_recv = g->ids_recv;
    if (w_recv) *w_recv = g->w_recv;
    if (y_recv) *y_recv = g->y_recv;
    return WISP_OK;
}

int wisp_ep_group_config(wisp_ep_group *g, int64_t wait_ns) {
    if (!g || wait_ns < 1000000) return fail(WISP_ERR_INVALID, "wisp_ep_group_config: wait limit below 1 ms");
    g->wait_ns = wait_ns;
    return WISP_OK;
}

int wisp_ep_dispatch(wisp_ep_group *g, const void *x, const void *topk_ids, int32_t ids_int64,
                     const float *topk_weights, int32_t num_tokens, int32_t top_k, int32_t experts_per_rank,
                     void *stream) {
    if (!g) return fail(WISP_ERR_INVALID, "wisp_ep_dispatch: NULL group");
    if (num_tokens < 0 || top_k < 1 || experts_per_rank < 1 || experts_per_rank > 1024)
        return fail(WISP_ERR_INVALID, "wisp_ep_dispatch: bad sizes (1 <= experts_per_rank <= 1024)");
    const long P = (long)num_tokens * top_k;
    if (P > g->max_pairs)
        return fail(WISP_ERR_INVALID, "wisp_ep_dispatch: " + std::to_string(P) +
                                          " (token, k) pairs exceed the group's max_pairs " +
                                          std::to_string(g->max_pairs));
    if (P > 0 && (!x || !topk_ids || !topk_weights)) return fail(WISP_ERR_INVALID, "wisp_ep_dispatch: NULL tensor");
    if (!g->d_peer || !g->peer[(g->rank + 1) % g->world])
        return fail(WISP_ERR_INVALID, "wisp_ep_dispatch: group not connected");
    std::lock_guard<std::mutex> lk(g->mu);
    Guard guard(g->dev);
    DispatchArgs a{};
    a.x = reinterpret_cast<const uint4 *>(x);
    a.ids = topk_ids;
    a.ids64 = ids_int64;
    a.w = topk_weights;
    a.P = (int)P;
    a.K = top_k;
    a.H8 = g->H / 8;
    a.e_local = experts_per_rank;
    a.world = g->world;
    a.rank = g->rank;
    a.max_pairs = g->max_pairs;
    a.epoch = ++g->epoch;
    g->e_local = experts_per_rank;
    a.peer = g->d_peer;
    a.off_inbox = g->lay.inbox;
    a.off_recs = g->lay.recs;
    a.off_recv = g->lay.recv;
    a.counter = g->d_counter;
    const size_t smem = sizeof(int) * (size_t)std::max<long>(P, 1);
    static bool attr_done[64] = {};
    if (g->dev < 64 && !attr_done[g->dev]) {
        WISP_CUDA_TRY(cudaFuncSetAttribute(ep_dispatch_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           (int)(sizeof(int) * kMaxPairsLimit)));
        attr_done[g->dev] = true;
    }
    ep_dispatch_kernel<<<grid_for(P, g->dev), kThreads, smem, reinterpret_cast<cudaStream_t>(stream)>>>(a);
    WISP_CUDA_TRY(cudaGetLastError());
    return WISP_OK;
}

int wisp_ep_receive(wisp_ep_group *g, int32_t class_min_pairs, void *stream, int32_t *counts_out,
                    int32_t *src_pairs_out, int32_t *total_out) {
    if (!g) return fail(WISP_ERR_INVALID, "wisp_ep_receive: NULL group");
    std::lock_guard<std::mutex> lk(g->mu);
    Guard guard(g->dev);
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    ReceiveArgs a{};
    a.base = g->base;
    a.off_inbox = g->lay.inbox;
    a.off_recs = g->lay.recs;
    a.off_recv = g->lay.recv;
    a.world = g->world;
    a.max_pairs = g->max_pairs;
    a.H8 = g->H / 8;
    a.epoch = g->epoch;
    a.e_local = g->e_local;
    a.class_min_pairs = class_min_pairs;
    a.wait_ns = g->wait_ns;
    a.x_recv = reinterpret_cast<uint4 *>(g->x_recv);
    a.ids_recv = g->ids_recv;
    a.map_recv = g->map_recv;
    a.w_recv = g->w_recv;
    a.info = g->d_info;
    const size_t smem = sizeof(int) * ((size_t)g->world * g->max_pairs + g->e_local);
    if (smem > g->recv_smem) {
        WISP_CUDA_TRY(cudaFuncSetAttribute(ep_receive_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
        g->recv_smem = smem;
    }
    g->h_info[0] = -1;
    ep_receive_kernel<<<grid_for((long)g->world * g->max_pairs, g->dev), kThreads, smem, s>>>(a);
    WISP_CUDA_TRY(cudaGetLastError());
    WISP_CUDA_TRY(cudaEventRecord(g->ev, s));
    WISP_CUDA_TRY(cudaEventSynchronize(g->ev));
    volatile int32_t *info = g->h_info;
    const int st = info[0];
    const int R = info[1];
    if (counts_out)
        for (int r = 0; r < g->world; ++r) counts_out[r] = info[2 + r];
    if (src_pairs_out)
        for (int r = 0; r < g->world; ++r) src_pairs_out[r] = info[2 + g->world + r];
    if (total_out) *total_out = R;
    g->last_R = st == WISP_OK ? R : 0;
    if (st == WISP_ERR_BAD_EXPERT)
        return fail(WISP_ERR_BAD_EXPERT, "wisp: a rank routed an expert id outside [0, experts_per_rank * world)");
    if (st == WISP_ERR_TIMEOUT)
        return fail(WISP_ERR_TIMEOUT, "wisp_ep_receive: a source's rows did not arrive within the wait limit");
    if (st != WISP_OK) return fail(WISP_ERR_CUDA, "wisp_ep_receive: receive kernel did not report");
    return WISP_OK;
}

int wisp_ep_return(wisp_ep_group *g, void *stream) {
    if (!g) return fail(WISP_ERR_INVALID, "wisp_ep_return: NULL group");
    std::lock_guard<std::mutex> lk(g->mu);
    Guard guard(g->dev);
    ReturnArgs a{};
    a.y_recv = reinterpret_cast<const uint4 *>(g->y_recv);
    a.map_recv = g->map_recv;
    a.R = g->last_R;
    a.H8 = g->H / 8;
    a.world = g->world;
    a.rank = g->rank;
    a.epoch = g->epoch;
    a.peer = g->d_peer;
    a.off_back = g->lay.back;
    a.off_back_flag = g->lay.back_flag;
    a.counter = g->d_counter + 1;
    ep_return_kernel<<<grid_for(a.R, g->dev), kThreads, 0, reinterpret_cast<cudaStream_t>(stream)>>>(a);
    WISP_CUDA_TRY(cudaGetLastError());
    return WISP_OK;
}

int wisp_ep_combine(wisp_ep_group *g, int32_t num_tokens, int32_t top_k, void *out, void *stream) {
    if (!g) return fail(WISP_ERR_INVALID, "wisp_ep_combine: NULL group");
    if (num_tokens < 0 || top_k < 1 || (long)num_tokens * top_k > g->max_pairs)
        return fail(WISP_ERR_INVALID, "wisp_ep_combine: bad sizes");
    if (num_tokens > 0 && !out) return fail(WISP_ERR_INVALID, "wisp_ep_combine: NULL out");
    std::lock_guard<std::mutex> lk(g->mu);
    Guard guard(g->dev);
    CombineArgs a{};
    a.base = g->base;
    a.off_back = g->lay.back;
    a.off_back_flag = g->lay.back_flag;
    a.world = g->world;
    a.T = num_tokens;
    a.K = top_k;
    a.H8 = g->H / 8;
    a.epoch = g->epoch;
    a.wait_ns = g->wait_ns;
    a.out = reinterpret_cast<uint4 *>(out);
    a.status = g->d_status;
    const long n = (long)num_tokens * a.H8;
    const int grid = (int)std::max<long>(1, std::min<long>((n + kThreads - 1) / kThreads, 296));
    ep_combine_kernel<<<grid, kThreads, 0, reinterpret_cast<cudaStream_t>(stream)>>>(a);
    WISP_CUDA_TRY(cudaGetLastError());
    return WISP_OK;
}

int wisp_ep_sync(wisp_ep_group *g) {
    if (!g) return fail(WISP_ERR_INVALID, "wisp_ep_sync: NULL group");
    std::lock_guard<std::mutex> lk(g->mu);
    Guard guard(g->dev);
    WISP_CUDA_TRY(cudaDeviceSynchronize());
    int st = 0;
    WISP_CUDA_TRY(cudaMemcpy(&st, g->d_status, sizeof(int), cudaMemcpyDeviceToHost));
    if (st == WISP_OK) return WISP_OK;
    const int zero = 0;
    WISP_CUDA_TRY(cudaMemcpy(g->d_status, &zero, sizeof(int), cudaMemcpyHostToDevice));
    if (st == WISP_ERR_TIMEOUT)
        return fail(st, "wisp: an expert-parallel wait ran past its limit (a rank did not take part)");
    return fail(st, "wisp: an expert-parallel call failed (status " + std::to_string(st) + ")");
}

}  // extern "C"
