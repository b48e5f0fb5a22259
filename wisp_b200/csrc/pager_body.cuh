// The device pager (K1) body: included by pager.cu (standalone pager kernel)
// and forward.cu (block 0 of the persistent forward kernel).
//
// One CTA of kPagerThreads threads runs one forward's bookkeeping: the
// first-fit token sub-batching of _wisp_forward_cuda_paged
// (src/wisp/integrations/vllm/fused_moe.py:1102-1140) and, for every group in
// order, the reference's ensure_resident LRU step (fused_moe.py:264-358),
// bit-exact:
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
// pager_body leaves the new LRU state in shared memory and writes what the
// compute needs (slot of every (t, k) pair, per-group unique-slot lists with
// their pairs, the device header); pager_finish then writes the LRU state
// back and publishes the page-in list to the host mailbox.  The forward
// kernel calls pager_finish only once every other block has finished reading
// the pre-call expert map (for its speculative start).
#pragma once
#include "common.cuh"
#include "pager.cuh"

namespace wisp {

namespace pager_detail {

constexpr int kThreads = kPagerThreads;
constexpr int kMaxMaskWords = 32;     // E <= 1024
constexpr int kLinearRun = 9;
constexpr int kPerturbShift = 5;
constexpr int kIdsInSmem = 2048;      // (t, k) pairs staged in shared memory up to this
constexpr int kGroupsInSmem = 2048;   // group starts kept in shared memory up to this

// Table size after inserting n keys one at a time (8 entries, grown to the
// smallest power of two above 4*used whenever 5*fill >= 3*mask).
__device__ __host__ inline int final_table_size(int n) {
    int size = 8;
    for (int used = 1; used <= n; ++used) {
        if (used * 5 >= (size - 1) * 3) {
            int ns = 8;
            while (ns <= used * 4) ns <<= 1;
            size = ns;
        }
    }
    return size;
}

static __device__ inline void tab_place(int16_t *tab, int mask, int key) {
    unsigned i = (unsigned)key & (unsigned)mask;
    unsigned perturb = (unsigned)key;
    while (true) {
        int run = (i + kLinearRun <= (unsigned)mask) ? kLinearRun : 0;
        for (int r = 0; r <= run; ++r) {
            if (tab[i + r] < 0) {
                tab[i + r] = (int16_t)key;
                return;
            }
        }
        perturb >>= kPerturbShift;
        i = (i * 5u + 1u + perturb) & (unsigned)mask;
    }
}

// Single-thread model of the interpreter's set: insert asc[0..n) in order,
// write the iteration order to order[] (also used as scratch while rehashing).
static __device__ void set_iteration_order(const int *asc, int n, int16_t *tab, int *order) {
    int size = 8, mask = 7;
    for (int s = 0; s < size; ++s) tab[s] = -1;
    for (int u = 0; u < n; ++u) {
        tab_place(tab, mask, asc[u]);
        int used = u + 1;
        if (used * 5 >= mask * 3) {
            int ns = 8;
            while (ns <= used * 4) ns <<= 1;
            int j = 0;
            for (int s = 0; s < size; ++s)
                if (tab[s] >= 0) order[j++] = tab[s];
            for (int s = 0; s < ns; ++s) tab[s] = -1;
            size = ns;
            mask = ns - 1;
            for (int q = 0; q < j; ++q) tab_place(tab, mask, order[q]);
        }
    }
    int j = 0;
    for (int s = 0; s < size; ++s)
        if (tab[s] >= 0) order[j++] = tab[s];
}

struct Scalars {
    long long clock, stat[4];
    int n, nm, nfree, need, G, status, err_group, mtotal, utotal, fast, nhit;
    uint32_t mask[kMaxMaskWords];
    uint32_t umask[kMaxMaskWords];  // union of the groups' needed sets (the forward's unique experts)
};

struct Smem {
    Scalars *sc;
    int64_t *tick;
    int *s2e, *lastg, *fresh, *fre, *emap, *asc, *order, *miss, *pos, *cnt, *fill, *uord;
    int *ids;   // staged ids (or nullptr)
    int *grp;   // group starts (shared or global)
    int16_t *tab;
};

__host__ __device__ inline bool ids_in_smem(int T, int K) { return (long)T * K <= kIdsInSmem; }
__host__ __device__ inline bool groups_in_smem(int T) { return T + 1 <= kGroupsInSmem; }

__device__ inline Smem carve(unsigned char *p, int E, int cap, int T, int K, int32_t *grp_global) {
    Smem S;
    S.sc = reinterpret_cast<Scalars *>(p); p += (sizeof(Scalars) + 15) & ~size_t(15);
    S.tick = reinterpret_cast<int64_t *>(p); p += sizeof(int64_t) * cap;
    S.s2e = reinterpret_cast<int *>(p); p += sizeof(int) * cap;
    S.lastg = reinterpret_cast<int *>(p); p += sizeof(int) * cap;
    S.fresh = reinterpret_cast<int *>(p); p += sizeof(int) * cap;
    S.fre = reinterpret_cast<int *>(p); p += sizeof(int) * cap;
    S.emap = reinterpret_cast<int *>(p); p += sizeof(int) * E;
    S.asc = reinterpret_cast<int *>(p); p += sizeof(int) * E;
    S.order = reinterpret_cast<int *>(p); p += sizeof(int) * E;
    S.miss = reinterpret_cast<int *>(p); p += sizeof(int) * E;
    S.pos = reinterpret_cast<int *>(p); p += sizeof(int) * E;
    S.fill = reinterpret_cast<int *>(p); p += sizeof(int) * E;
    S.uord = reinterpret_cast<int *>(p); p += sizeof(int) * E;
    S.cnt = reinterpret_cast<int *>(p); p += sizeof(int) * (E + 1);
    S.ids = nullptr;
    if (ids_in_smem(T, K)) {
        S.ids = reinterpret_cast<int *>(p);
        p += sizeof(int) * ((size_t)T * K);
    }
    S.grp = grp_global;
    if (groups_in_smem(T)) {
        S.grp = reinterpret_cast<int *>(p);
        p += sizeof(int) * ((size_t)T + 1);
    }
    S.tab = reinterpret_cast<int16_t *>(p);
    return S;
}

__host__ __device__ inline size_t smem_bytes(int E, int cap, int T, int K) {
    size_t b = (sizeof(Scalars) + 15) & ~size_t(15);
    b += sizeof(int64_t) * cap;                  // tick
    b += sizeof(int) * (size_t)cap * 4;          // s2e, lastg, fresh, free
    b += sizeof(int) * (size_t)E * 7;            // emap, asc, order, miss, pos, fill, uord
    b += sizeof(int) * (size_t)(E + 1);          // cnt
    if (ids_in_smem(T, K)) b += sizeof(int) * ((size_t)T * K);
    if (groups_in_smem(T)) b += sizeof(int) * ((size_t)T + 1);
    b += sizeof(int16_t) * (size_t)final_table_size(E) + 16;
    return (b + 15) & ~size_t(15);
}

}  // namespace pager_detail

using namespace pager_detail;

static __device__ __forceinline__ int pager_id(const PagerParams &a, const Smem &S, long p) {
    return S.ids ? S.ids[p] : (int)load_id64(a.ids, a.ids64, p);
}

// All threads of one CTA (any multiple of 32, at least kThreads).  On return
// the new state is in shared memory (smem_raw) and the compute outputs are in
// device memory.
static __device__ __noinline__ void pager_body(const PagerParams &a, unsigned char *smem_raw) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int nth = blockDim.x;
    const int E = a.E, cap = a.cap, K = a.K, T = a.T;
    const Smem S = carve(smem_raw, E, cap, T, K, a.grp_start);
    Scalars &sc = *S.sc;
    int *mb_miss = a.mb + mailbox_miss_offset(T);

    // ---- load state and ids ---------------------------------------------------
    for (int s = tid; s < cap; s += nth) {
        S.tick[s] = a.tick[s];
        S.s2e[s] = a.s2e[s];
        S.lastg[s] = -1;
        S.fresh[s] = 0;
    }
    for (int e = tid; e < E; e += nth) S.emap[e] = a.emap[e];
    if (tid < kMaxMaskWords) sc.umask[tid] = 0;
    int bad = 0;
    if (S.ids) {
        for (long p = tid; p < (long)T * K; p += nth) {
            const long long e = load_id64(a.ids, a.ids64, p);
            bad |= (e < 0 || e >= E);
            S.ids[p] = (int)e;
        }
    } else {
        for (long p = tid; p < (long)T * K; p += nth) {
            const long long e = load_id64(a.ids, a.ids64, p);
            bad |= (e < 0 || e >= E);
        }
    }
    if (tid == 0) {
        sc.clock = a.hdr[0];
        for (int i = 0; i < 4; ++i) sc.stat[i] = a.hdr[1 + i];
        sc.status = WISP_OK;
        sc.err_group = -1;
        sc.mtotal = 0;
        sc.utotal = 0;
    }
    if (__syncthreads_or(bad)) {
        if (tid == 0) {
            sc.status = WISP_ERR_BAD_EXPERT;
            sc.G = 0;
        }
        goto finish;
    }

    // ---- phase A: first-fit groups (warp 0) ------------------------------------
    if (warp == 0) {
        int G = 0;
        if (a.single_group || a.mode == WISP_MODE_RESIDENT) {
            if (lane == 0) S.grp[0] = 0;
            G = 1;
        } else {
            uint32_t cur = 0;
            int start = 0;
            for (int t = 0; t < T; ++t) {
                uint32_t tw = 0;
                for (int j = 0; j < K; ++j) {
                    const int e = pager_id(a, S, (long)t * K + j);
                    if ((e >> 5) == lane) tw |= 1u << (e & 31);
                }
                const uint32_t merged = cur | tw;
                const int c = __reduce_add_sync(0xffffffffu, __popc(merged));
                if (c <= cap || t == start) {
                    cur = merged;
                } else {
                    if (lane == 0) S.grp[G] = start;
                    ++G;
                    start = t;
                    cur = tw;
                }
            }
            if (lane == 0) S.grp[G] = start;
            ++G;
        }
        if (lane == 0) {
            S.grp[G] = T;
            sc.G = G;
        }
    }
    __syncthreads();
    if (a.count_forward && tid == 0) sc.stat[0] += 1;

    // ---- phase B: one LRU step per group --------------------------------------------
    for (int g = 0; g < sc.G; ++g) {
        const int t0 = S.grp[g], t1 = S.grp[g + 1];
        const long p0 = (long)t0 * K, p1 = (long)t1 * K;
        if (tid < kMaxMaskWords) sc.mask[tid] = 0;
        __syncthreads();
        for (long p = p0 + tid; p < p1; p += nth) {
            const int e = pager_id(a, S, p);
            atomicOr(&sc.mask[e >> 5], 1u << (e & 31));
        }
        __syncthreads();
        if (tid < kMaxMaskWords) sc.umask[tid] |= sc.mask[tid];
        // ascending needed list
        if (warp == 0) {
            uint32_t w = (lane < kMaxMaskWords) ? sc.mask[lane] : 0u;
            const int c = __popc(w);
            int incl = c;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int v = __shfl_up_sync(0xffffffffu, incl, o);
                if (lane >= o) incl += v;
            }
            int base = incl - c;
            while (w) {
                const int b = __ffs(w) - 1;
                w &= w - 1;
                S.asc[base++] = lane * 32 + b;
            }
            if (lane == 31) sc.n = incl;
        }
        __syncthreads();
        const int n = sc.n;
        if (a.mode == WISP_MODE_RESIDENT) {
            // identity scratch: no LRU bookkeeping (fused_moe.py:974-976)
            if (tid == 0) sc.nm = 0;
            __syncthreads();
        } else {
            // needed set in interpreter order
            if (tid == 0) {
                const int fs = final_table_size(n);
                sc.fast = (n == 0 || S.asc[n - 1] < fs) ? 1 : 0;
                if (!sc.fast) set_iteration_order(S.asc, n, S.tab, S.order);
            }
            __syncthreads();
            const int* order = sc.fast ? S.asc : S.order;
            // missing list in that order
            if (warp == 0) {
                int nm = 0;
                for (int base = 0; base < n; base += 32) {
                    const int i = base + lane;
                    const bool m = (i < n) && (S.emap[order[i]] < 0);
                    const unsigned bal = __ballot_sync(0xffffffffu, m);
                    if (m) S.miss[nm + __popc(bal & ((1u << lane) - 1u))] = order[i];
                    nm += __popc(bal);
                }
                if (lane == 0) {
                    sc.nm = nm;
                    sc.stat[2] += n - nm;  // hits
                }
            }
            __syncthreads();
        }
        const int nm = sc.nm;
        if (a.mode != WISP_MODE_RESIDENT) {
            if (nm > 0) {
                // free slots ascending; eviction candidates
                if (warp == 0) {
                    int nf = 0, nc = 0;
                    for (int base = 0; base < cap; base += 32) {
                        const int s = base + lane;
                        const bool f = (s < cap) && (S.s2e[s] < 0);
                        bool c = false;
                        if (s < cap && S.s2e[s] >= 0) {
                            const int e = S.s2e[s];
                            c = !((sc.mask[e >> 5] >> (e & 31)) & 1u);
                        }
                        const unsigned bf = __ballot_sync(0xffffffffu, f);
                        const unsigned bc = __ballot_sync(0xffffffffu, c);
                        if (f) S.fre[nf + __popc(bf & ((1u << lane) - 1u))] = s;
                        nf += __popc(bf);
                        nc += __popc(bc);
                    }
                    if (lane == 0) {
                        sc.nfree = nf;
                        sc.need = nm - nf;
                        if (nm - nf > nc) {
                            sc.status = WISP_ERR_OVERFLOW;
                            sc.err_group = g;
                        }
                    }
                }
                __syncthreads();
                if (sc.status != WISP_OK) break;
                const int nfree = sc.nfree, need = sc.need;
                if (need > 0) {
                    // rank each candidate by (tick, slot); the first `need` are victims
                    for (int s = tid; s < cap; s += nth) {
                        const int e = S.s2e[s];
                        if (e < 0 || ((sc.mask[e >> 5] >> (e & 31)) & 1u)) continue;
                        const long long ts = S.tick[s];
                        int rank = 0;
                        for (int q = 0; q < cap; ++q) {
                            const int eq = S.s2e[q];
                            if (eq < 0 || ((sc.mask[eq >> 5] >> (eq & 31)) & 1u)) continue;
                            const long long tq = S.tick[q];
                            rank += (tq < ts) || (tq == ts && q < s);
                        }
                        if (rank < need) S.fre[nfree + rank] = s;
                    }
                    __syncthreads();
                    for (int r = tid; r < need; r += nth) {
                        const int s = S.fre[nfree + r];
                        S.emap[S.s2e[s]] = -1;
                        S.s2e[s] = -1;
                    }
                    if (tid == 0) sc.stat[3] += need;  // evictions
                    __syncthreads();
                }
                const int total_free = nfree + (need > 0 ? need : 0);
                if (tid == 0) sc.clock += 1;
                __syncthreads();
                const long long clk = sc.clock;
                const int mbase = sc.mtotal;
                for (int i = tid; i < nm; i += nth) {
                    const int e = S.miss[i];
                    const int s = S.fre[total_free - 1 - i];  // LIFO pop
                    S.emap[e] = s;
                    S.s2e[s] = e;
                    S.tick[s] = clk;
                    const uint32_t gen = a.slot_gen[s] + 1;  // slots are distinct within a group
                    a.slot_gen[s] = gen;
                    S.fresh[s] = 1;
                    int *rec = mb_miss + kMbRec * (mbase + i);
                    rec[0] = e;
                    rec[1] = s;
                    rec[2] = g;
                    rec[3] = S.lastg[s];
                    rec[4] = (int)gen;
                }
                if (tid == 0) {
                    sc.stat[1] += nm;  // misses
                    sc.mtotal = mbase + nm;
                }
                __syncthreads();
            } else {
                if (tid == 0) sc.clock += 1;
                __syncthreads();
            }
            const long long clk = sc.clock;
            for (int i = tid; i < n; i += nth) {
                const int s = S.emap[S.asc[i]];
                S.tick[s] = clk;
                S.lastg[s] = g;
            }
        }
        // unique order for the compute: hits (ascending id), then the misses in
        // page-in order, so work on resident experts starts first
        if (warp == 0) {
            int nh = 0;
            for (int base = 0; base < n; base += 32) {
                const int i = base + lane;
                const int e = (i < n) ? S.asc[i] : -1;
                bool missed = false;
                if (e >= 0)
                    for (int q = 0; q < nm; ++q) missed |= (S.miss[q] == e);
                const bool h = (e >= 0) && !missed;
                const unsigned bal = __ballot_sync(0xffffffffu, h);
                if (h) S.uord[nh + __popc(bal & ((1u << lane) - 1u))] = e;
                nh += __popc(bal);
            }
            if (lane == 0) sc.nhit = nh;
        }
        __syncthreads();
        for (int i = tid; i < nm; i += nth) S.uord[sc.nhit + i] = S.miss[i];
        __syncthreads();
        // per-(t,k) slots and per-group unique-slot CSR for the compute kernels
        for (int i = tid; i < n; i += nth) {
            const int e = S.uord[i];
            S.pos[e] = i;
            S.cnt[i] = 0;
            S.fill[i] = 0;
            const int s = S.emap[e];
            a.u_slot[p0 + i] = s;
            // a slot filled before this call is complete (that call's compute
            // waited for it): 0 = no wait; else the generation to wait for
            a.u_gen[p0 + i] = S.fresh[s] ? (int)a.slot_gen[s] : 0;
        }
        __syncthreads();
        for (long p = p0 + tid; p < p1; p += nth) {
            const int e = pager_id(a, S, p);
            a.slots[p] = S.emap[e];
            atomicAdd(&S.cnt[S.pos[e]], 1);
        }
        __syncthreads();
        if (warp == 0) {
            int run = 0;
            for (int base = 0; base < n; base += 32) {
                const int i = base + lane;
                const int c = (i < n) ? S.cnt[i] : 0;
                int incl = c;
#pragma unroll
                for (int o = 1; o < 32; o <<= 1) {
                    const int v = __shfl_up_sync(0xffffffffu, incl, o);
                    if (lane >= o) incl += v;
                }
                if (i < n) {
                    a.u_off[p0 + g + i] = run + incl - c;
                    S.cnt[i] = run + incl - c;  // now the exclusive offset
                }
                run += __shfl_sync(0xffffffffu, incl, 31);
            }
            if (lane == 0) a.u_off[p0 + g + n] = run;
        }
        __syncthreads();
        for (long p = p0 + tid; p < p1; p += nth) {
            const int i = S.pos[pager_id(a, S, p)];
            const int at = atomicAdd(&S.fill[i], 1);
            a.u_pairs[p0 + S.cnt[i] + at] = (int)p;
        }
        if (tid == 0) {
            a.grp_nu[g] = n;
            a.grp_nhit[g] = sc.nhit;
            sc.utotal += n;
        }
        __syncthreads();
    }
finish:
    __syncthreads();
    if (tid == 0) {
        a.dev_hdr[kHdrStatus] = sc.status;
        a.dev_hdr[kHdrGroups] = sc.G;
        a.dev_hdr[kHdrMisses] = sc.mtotal;
        a.dev_hdr[kHdrUnique] = sc.utotal;
    }
    if (S.grp != a.grp_start)
        for (int g = tid; g <= sc.G; g += nth) a.grp_start[g] = S.grp[g];
    __threadfence();  // every thread's outputs visible device-wide before the CTA moves on
    __syncthreads();
}

// After pager_body (same CTA, shared memory untouched since): write the LRU
// state back and publish the groups and the page-in list to the mailbox.
static __device__ __noinline__ void pager_finish(const PagerParams &a, unsigned char *smem_raw,
                                                 bool publish) {
    const int tid = threadIdx.x, nth = blockDim.x;
    const int E = a.E, cap = a.cap, T = a.T;
    const Smem S = carve(smem_raw, E, cap, T, a.K, a.grp_start);
    const Scalars &sc = *S.sc;
    if (sc.status == WISP_OK || sc.status == WISP_ERR_OVERFLOW) {
        for (int s = tid; s < cap; s += nth) {
            a.tick[s] = S.tick[s];
            a.s2e[s] = S.s2e[s];
        }
        for (int e = tid; e < E; e += nth) a.emap[e] = S.emap[e];
        // the forward's unique experts (fused_moe.py:1170-1176); a resident
        // forward leaves them alone, as the reference's does
        if (a.last_unique && a.count_forward && a.mode != WISP_MODE_RESIDENT && sc.status == WISP_OK)
            for (int w = tid; w < (E + 31) / 32; w += nth) a.last_unique[w] = sc.umask[w];
        if (tid == 0) {
            a.hdr[0] = sc.clock;
            for (int i = 0; i < 4; ++i) a.hdr[1 + i] = sc.stat[i];
            a.hdr[5] += sc.G;       // telemetry: groups run
            a.hdr[6] += sc.utotal;  // telemetry: unique experts read, summed over groups
        }
    }
    if (publish) {
        int *mb_grp = a.mb + kMbHeader;
        int *mb_nu = mb_grp + (T + 1);
        const int G = sc.status == WISP_OK ? sc.G : 0;
        for (int w = tid; w < kMaxMaskWords; w += nth) a.mb[kMbUnique + w] = (int)sc.umask[w];
        for (int g = tid; g <= G; g += nth) mb_grp[g] = S.grp[g];
        for (int g = tid; g < G; g += nth) mb_nu[g] = a.grp_nu[g];
        __syncthreads();
        if (tid == 0) {
            a.mb[1] = sc.G;
            a.mb[2] = sc.mtotal;
            a.mb[3] = sc.err_group;
            a.mb[4] = sc.utotal;
            a.mb[0] = sc.status;
            __threadfence_system();  // the records and the header before the sequence number
            a.mb[7] = (int)a.seq;
            __threadfence_system();
        }
    }
    __syncthreads();
}

}  // namespace wisp
