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
#include "common.cuh"
#include "pager.cuh"

namespace wisp {

namespace {

constexpr int kThreads = 256;
constexpr int kMaxMaskWords = 32;  // E <= 1024
constexpr int kLinearRun = 9;
constexpr int kPerturbShift = 5;

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

__device__ inline void tab_place(int16_t *tab, int mask, int key) {
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
// write the iteration order to order[].  tmp has room for n entries.
__device__ void set_iteration_order(const int *asc, int n, int16_t *tab, int *order) {
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

struct Smem {
    int64_t *tick;
    int *s2e, *lastg, *fre, *emap, *asc, *order, *miss, *pos, *cnt, *fill;
    int16_t *tab;
};

}  // namespace

size_t pager_smem_bytes(int E, int cap) {
    size_t b = 0;
    b += sizeof(int64_t) * cap;                  // tick
    b += sizeof(int) * (size_t)cap * 3;          // s2e, lastg, free
    b += sizeof(int) * (size_t)E * 6;            // emap, asc, order, miss, pos, fill
    b += sizeof(int) * (size_t)(E + 1);          // cnt
    b += sizeof(int16_t) * (size_t)final_table_size(E) + 16;
    return (b + 15) & ~size_t(15);
}

__global__ void __launch_bounds__(kThreads, 1) pager_kernel(PagerParams a) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    __shared__ uint32_t s_mask[kMaxMaskWords];
    __shared__ int s_n, s_nm, s_nfree, s_ncand, s_need, s_G, s_status, s_err_group, s_mtotal,
        s_utotal, s_fast;
    __shared__ long long s_clock, s_stat[4];

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int E = a.E, cap = a.cap, K = a.K, T = a.T;

    Smem S;
    {
        unsigned char *p = smem_raw;
        S.tick = reinterpret_cast<int64_t *>(p); p += sizeof(int64_t) * cap;
        S.s2e = reinterpret_cast<int *>(p); p += sizeof(int) * cap;
        S.lastg = reinterpret_cast<int *>(p); p += sizeof(int) * cap;
        S.fre = reinterpret_cast<int *>(p); p += sizeof(int) * cap;
        S.emap = reinterpret_cast<int *>(p); p += sizeof(int) * E;
        S.asc = reinterpret_cast<int *>(p); p += sizeof(int) * E;
        S.order = reinterpret_cast<int *>(p); p += sizeof(int) * E;
        S.miss = reinterpret_cast<int *>(p); p += sizeof(int) * E;
        S.pos = reinterpret_cast<int *>(p); p += sizeof(int) * E;
        S.fill = reinterpret_cast<int *>(p); p += sizeof(int) * E;
        S.cnt = reinterpret_cast<int *>(p); p += sizeof(int) * (E + 1);
        S.tab = reinterpret_cast<int16_t *>(p);
    }
    int *mb_grp = a.mb + kMbHeader;
    int *mb_nu = mb_grp + (T + 1);
    int *mb_miss = a.mb + mailbox_miss_offset(T);

    // ---- load state -------------------------------------------------------
    for (int s = tid; s < cap; s += kThreads) {
        S.tick[s] = a.tick[s];
        S.s2e[s] = a.s2e[s];
        S.lastg[s] = -1;
    }
    for (int e = tid; e < E; e += kThreads) S.emap[e] = a.emap[e];
    if (tid == 0) {
        s_clock = a.hdr[0];
        for (int i = 0; i < 4; ++i) s_stat[i] = a.hdr[1 + i];
        s_status = WISP_OK;
        s_err_group = -1;
        s_mtotal = 0;
        s_utotal = 0;
    }

    // ---- phase A: validate ids, first-fit groups (warp 0) -------------------
    if (warp == 0) {
        bool bad = false;
        int G = 0;
        if (a.single_group || a.mode == WISP_MODE_RESIDENT) {
            for (long p = lane; p < (long)T * K; p += 32) {
                long long e = load_id64(a.ids, a.ids64, p);
                bad |= (e < 0 || e >= E);
            }
            if (lane == 0) a.grp_start[0] = 0;
            G = 1;
        } else {
            uint32_t cur = 0;
            int start = 0;
            for (int t = 0; t < T; ++t) {
                uint32_t tw = 0;
                for (int j = 0; j < K; ++j) {
                    long long e = load_id64(a.ids, a.ids64, (long)t * K + j);
                    if (e < 0 || e >= E) {
                        bad = true;
                    } else if ((int)(e >> 5) == lane) {
                        tw |= 1u << (e & 31);
                    }
                }
                uint32_t merged = cur | tw;
                int c = __reduce_add_sync(0xffffffffu, __popc(merged));
                if (c <= cap || t == start) {
                    cur = merged;
                } else {
                    if (lane == 0) a.grp_start[G] = start;
                    ++G;
                    start = t;
                    cur = tw;
                }
            }
            if (lane == 0) a.grp_start[G] = start;
            ++G;
        }
        bad = __any_sync(0xffffffffu, bad);
        if (lane == 0) {
            a.grp_start[G] = T;
            s_G = G;
            if (bad) s_status = WISP_ERR_BAD_EXPERT;
        }
    }
    __syncthreads();
    if (s_status != WISP_OK) goto finish_nostate;
    if (a.count_forward && tid == 0) s_stat[0] += 1;

    // ---- phase B: one LRU step per group ------------------------------------
    for (int g = 0; g < s_G; ++g) {
        const int t0 = a.grp_start[g], t1 = a.grp_start[g + 1];
        const long p0 = (long)t0 * K, p1 = (long)t1 * K;
        if (tid < kMaxMaskWords) s_mask[tid] = 0;
        __syncthreads();
        for (long p = p0 + tid; p < p1; p += kThreads) {
            int e = (int)load_id64(a.ids, a.ids64, p);
            atomicOr(&s_mask[e >> 5], 1u << (e & 31));
        }
        __syncthreads();
        // ascending needed list + expert -> index
        if (warp == 0) {
            uint32_t w = (lane < kMaxMaskWords) ? s_mask[lane] : 0u;
            int c = __popc(w);
            int incl = c;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                int v = __shfl_up_sync(0xffffffffu, incl, o);
                if (lane >= o) incl += v;
            }
            int base = incl - c;
            while (w) {
                int b = __ffs(w) - 1;
                w &= w - 1;
                int e = lane * 32 + b;
                S.asc[base] = e;
                S.pos[e] = base;
                ++base;
            }
            if (lane == 31) s_n = incl;
        }
        __syncthreads();
        const int n = s_n;
        if (a.mode == WISP_MODE_RESIDENT) {
            // identity scratch: no LRU bookkeeping (fused_moe.py:974-976)
            for (int i = tid; i < n; i += kThreads) S.order[i] = S.asc[i];
            if (tid == 0) { s_nm = 0; }
            __syncthreads();
        } else {
            // needed set in interpreter order
            if (tid == 0) {
                int fs = final_table_size(n);
                s_fast = (n == 0 || S.asc[n - 1] < fs) ? 1 : 0;
                if (!s_fast) set_iteration_order(S.asc, n, S.tab, S.order);
            }
            __syncthreads();
            if (s_fast)
                for (int i = tid; i < n; i += kThreads) S.order[i] = S.asc[i];
            __syncthreads();
            // missing list in that order
            if (warp == 0) {
                int nm = 0;
                for (int base = 0; base < n; base += 32) {
                    int i = base + lane;
                    bool m = (i < n) && (S.emap[S.order[i]] < 0);
                    unsigned bal = __ballot_sync(0xffffffffu, m);
                    if (m) S.miss[nm + __popc(bal & ((1u << lane) - 1u))] = S.order[i];
                    nm += __popc(bal);
                }
                if (lane == 0) {
                    s_nm = nm;
                    s_stat[2] += n - nm;  // hits
                }
            }
            __syncthreads();
        }
        const int nm = s_nm;
        if (a.mode != WISP_MODE_RESIDENT) {
            if (nm > 0) {
                // free slots ascending; eviction candidates
                if (warp == 0) {
                    int nf = 0, nc = 0;
                    for (int base = 0; base < cap; base += 32) {
                        int s = base + lane;
                        bool f = (s < cap) && (S.s2e[s] < 0);
                        bool c = false;
                        if (s < cap && S.s2e[s] >= 0) {
                            int e = S.s2e[s];
                            c = !((s_mask[e >> 5] >> (e & 31)) & 1u);
                        }
                        unsigned bf = __ballot_sync(0xffffffffu, f);
                        unsigned bc = __ballot_sync(0xffffffffu, c);
                        if (f) S.fre[nf + __popc(bf & ((1u << lane) - 1u))] = s;
                        nf += __popc(bf);
                        nc += __popc(bc);
                    }
                    if (lane == 0) {
                        s_nfree = nf;
                        s_ncand = nc;
                        s_need = nm - nf;
                        if (nm - nf > nc) {
                            s_status = WISP_ERR_OVERFLOW;
                            s_err_group = g;
                        }
                    }
                }
                __syncthreads();
                if (s_status != WISP_OK) break;
                const int nfree = s_nfree, need = s_need;
                if (need > 0) {
                    // rank each candidate by (tick, slot); the first `need` are victims
                    for (int s = tid; s < cap; s += kThreads) {
                        int e = S.s2e[s];
                        if (e < 0 || ((s_mask[e >> 5] >> (e & 31)) & 1u)) continue;
                        long long ts = S.tick[s];
                        int rank = 0;
                        for (int q = 0; q < cap; ++q) {
                            int eq = S.s2e[q];
                            if (eq < 0 || ((s_mask[eq >> 5] >> (eq & 31)) & 1u)) continue;
                            long long tq = S.tick[q];
                            rank += (tq < ts) || (tq == ts && q < s);
                        }
                        if (rank < need) S.fre[nfree + rank] = s;
                    }
                    __syncthreads();
                    for (int r = tid; r < need; r += kThreads) {
                        int s = S.fre[nfree + r];
                        S.emap[S.s2e[s]] = -1;
                        S.s2e[s] = -1;
                    }
                    if (tid == 0) s_stat[3] += need;  // evictions
                    __syncthreads();
                }
                const int total_free = nfree + (need > 0 ? need : 0);
                if (tid == 0) s_clock += 1;
                __syncthreads();
                const long long clk = s_clock;
                const int mbase = s_mtotal;
                for (int i = tid; i < nm; i += kThreads) {
                    int e = S.miss[i];
                    int s = S.fre[total_free - 1 - i];  // LIFO pop
                    S.emap[e] = s;
                    S.s2e[s] = e;
                    S.tick[s] = clk;
                    int *rec = mb_miss + 4 * (mbase + i);
                    rec[0] = e;
                    rec[1] = s;
                    rec[2] = g;
                    rec[3] = S.lastg[s];
                }
                if (tid == 0) {
                    s_stat[1] += nm;  // misses
                    s_mtotal = mbase + nm;
                }
                __syncthreads();
            } else {
                if (tid == 0) s_clock += 1;
                __syncthreads();
            }
            const long long clk = s_clock;
            for (int i = tid; i < n; i += kThreads) {
                int s = S.emap[S.asc[i]];
                S.tick[s] = clk;
                S.lastg[s] = g;
            }
        }
        // per-(t,k) slots and per-group unique-slot CSR for the compute kernels
        for (int i = tid; i < n; i += kThreads) {
            S.cnt[i] = 0;
            S.fill[i] = 0;
            a.u_slot[p0 + i] = S.emap[S.asc[i]];
        }
        __syncthreads();
        for (long p = p0 + tid; p < p1; p += kThreads) {
            int e = (int)load_id64(a.ids, a.ids64, p);
            a.slots[p] = S.emap[e];
            atomicAdd(&S.cnt[S.pos[e]], 1);
        }
        __syncthreads();
        if (warp == 0) {
            int run = 0;
            for (int base = 0; base < n; base += 32) {
                int i = base + lane;
                int c = (i < n) ? S.cnt[i] : 0;
                int incl = c;
#pragma unroll
                for (int o = 1; o < 32; o <<= 1) {
                    int v = __shfl_up_sync(0xffffffffu, incl, o);
                    if (lane >= o) incl += v;
                }
                if (i < n) a.u_off[p0 + g + i] = run + incl - c;
                run += __shfl_sync(0xffffffffu, incl, 31);
            }
            if (lane == 0) a.u_off[p0 + g + n] = run;
        }
        __syncthreads();
        for (long p = p0 + tid; p < p1; p += kThreads) {
            int e = (int)load_id64(a.ids, a.ids64, p);
            int i = S.pos[e];
            int at = atomicAdd(&S.fill[i], 1);
            a.u_pairs[p0 + a.u_off[p0 + g + i] + at] = (int)p;
        }
        if (tid == 0) {
            a.grp_nu[g] = n;
            mb_nu[g] = n;
            mb_grp[g] = t0;
            s_utotal += n;
        }
        __syncthreads();
    }

    // ---- write back ---------------------------------------------------------
    for (int s = tid; s < cap; s += kThreads) {
        a.tick[s] = S.tick[s];
        a.s2e[s] = S.s2e[s];
    }
    for (int e = tid; e < E; e += kThreads) a.emap[e] = S.emap[e];
    if (tid == 0) {
        a.hdr[0] = s_clock;
        for (int i = 0; i < 4; ++i) a.hdr[1 + i] = s_stat[i];
    }
finish_nostate:
    __syncthreads();
    if (tid == 0) {
        mb_grp[s_G] = T;
        a.mb[1] = s_G;
        a.mb[2] = s_mtotal;
        a.mb[3] = s_err_group;
        a.mb[4] = s_utotal;
        __threadfence_system();
        a.mb[0] = s_status;
    }
}

int launch_pager(const PagerParams &p, cudaStream_t stream) {
    const size_t smem = pager_smem_bytes(p.E, p.cap);
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
