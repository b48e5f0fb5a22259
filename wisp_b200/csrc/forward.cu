// Persistent cooperative forward kernel: one launch per layer forward.
//
//   phase 0  block 0 runs the LRU pager (pager_body) for every token group of
//            the call.  Meanwhile, when the call's experts fit the cap (one
//            group, decode sizes), the other blocks already run phase 1 for
//            the experts that were resident before the call: those are exactly
//            the pager's hits, they keep their slots, and block 0 writes the
//            new expert map back only after the first grid barrier;
//   then, per group g (work is handed out per warp, round-robin):
//   phase 1  gate-up GEMV + SiLU-mul, unit = one row pair of one unique
//            expert (the rest of them, after a speculative start); a unit of
//            an expert paged in during this call first waits until the slot's
//            generation flag (written by the copy stream after the two
//            copies) reaches the generation the pager assigned;
//   phase 2  down GEMV x routing weight, unit = four rows of one expert; the
//            last unit of a row quad to finish (arrival counter) sums the
//            group's tokens over k in routing order for those rows;
//            between groups block 0 publishes "group g done" to mapped host
//            memory, which lets the host copy thread overwrite slots g read.
//
// Decode-sized groups keep their unique-expert lists in shared memory and
// each warp loads the weights of its next unit while computing the current
// one; larger groups use the generic bodies of moe_body.cuh.  The arithmetic
// per (token, expert) pair is the same everywhere (moe_body.cuh documents it).
//
// Every wait (grid barrier, slot flag) is bounded by wait_ns of
// %globaltimer time; a wait that runs out sets the abort word and the sticky
// status WISP_ERR_TIMEOUT, every other wait then gives up too, and the
// kernel returns.
#include "forward.cuh"
#include "moe_body.cuh"
#include "pager_body.cuh"

namespace wisp {

namespace {

constexpr int kFwdThreads = kPagerThreads;  // 256: block 0 must run the pager
constexpr int kWarpsPerBlock = kFwdThreads / 32;
constexpr int kBlocksPerSm = 1;             // weight batches are held in registers
constexpr int kMetaU = 256;                 // unique experts in the shared-memory lists
constexpr int kMetaP = 256;                 // (token, k) pairs in the shared-memory lists
constexpr int kSpecMaxPairs = kMetaP;
constexpr int kGuChunks = 8;                // pipelined gate-up: H <= 8 * 256
constexpr int kDqChunks = 4;                // pipelined down: I <= 4 * 256

__device__ __forceinline__ void set_status(unsigned int *bar, int code) {
    atomicCAS(bar + kBarStatus, 0u, (unsigned)code);
}

// All blocks; returns false when the kernel is aborting.
__device__ bool grid_barrier(unsigned int *bar, long long wait_ns) {
    __shared__ int s_ok;
    __syncthreads();
    if (threadIdx.x == 0) {
        volatile unsigned int *vgen = bar + kBarGen;
        volatile unsigned int *vabort = bar + kBarAbort;
        int ok = 1;
        const unsigned int gen = *vgen;
        __threadfence();
        const unsigned int arrived = atomicAdd(bar + kBarArrive, 1u);
        if (arrived == gridDim.x - 1) {
            atomicExch(bar + kBarArrive, 0u);
            __threadfence();
            atomicAdd(bar + kBarGen, 1u);
        } else {
            const unsigned long long t0 = globaltimer_ns();
            while (*vgen == gen) {
                if (*vabort) break;
                if ((long long)(globaltimer_ns() - t0) > wait_ns) {
                    set_status(bar, WISP_ERR_TIMEOUT);
                    atomicExch(bar + kBarAbort, 1u);
                    break;
                }
                __nanosleep(32);
            }
        }
        if (*vabort) ok = 0;
        __threadfence();
        s_ok = ok;
    }
    __syncthreads();
    return s_ok != 0;
}

// One lane: wait until slot `slot` holds page-in generation `need`.
__device__ bool wait_slot(const uint32_t *ready, int slot, uint32_t need, unsigned int *bar,
                          long long wait_ns) {
    volatile const uint32_t *f = ready + slot;
    if ((int)(*f - need) >= 0) return true;
    volatile unsigned int *vabort = bar + kBarAbort;
    const unsigned long long t0 = globaltimer_ns();
    while ((int)(*f - need) < 0) {
        if (*vabort) return false;
        if ((long long)(globaltimer_ns() - t0) > wait_ns) {
            set_status(bar, WISP_ERR_TIMEOUT);
            atomicExch(bar + kBarAbort, 1u);
            return false;
        }
        __nanosleep(128);
    }
    __threadfence();
    return true;
}

// Per-block unique-expert lists of one group (shared memory).
struct Meta {
    int nu, maxnp;
    int slot[kMetaU], gen[kMetaU], off[kMetaU + 1];
    int pair[kMetaP], tok[kMetaP];
};

// ---- pipelined gate-up (decode sizes) ----------------------------------------
__device__ __forceinline__ void gu_load(const GroupCompute &a, int slot, int j, int lane,
                                        uint4 (&wg)[kGuChunks], uint4 (&wu)[kGuChunks]) {
    const int H = a.H, I = a.I;
    const __nv_bfloat16 *grow = a.w13 + (size_t)slot * (size_t)(2 * I) * H + (size_t)j * H;
    const __nv_bfloat16 *urow = grow + (size_t)I * H;
#pragma unroll
    for (int m = 0; m < kGuChunks; ++m) {
        const int c = m * 256 + lane * 8;
        if (c < H) {
            wg[m] = ld_cg16(grow + c);
            wu[m] = ld_cg16(urow + c);
        }
    }
}

template <int MAXP>
__device__ __forceinline__ void gu_compute(const GroupCompute &a, const Meta &m, int u, int j,
                                           int lane, const uint4 (&wg)[kGuChunks],
                                           const uint4 (&wu)[kGuChunks]) {
    const int H = a.H, I = a.I;
    const int q0 = m.off[u], q1 = m.off[u + 1];
    for (int qb = q0; qb < q1; qb += MAXP) {  // more pairs than MAXP: further passes, same registers
        const int np = min(MAXP, q1 - qb);
        float ag[MAXP], au[MAXP];
#pragma unroll
        for (int i = 0; i < MAXP; ++i) {
            ag[i] = 0.f;
            au[i] = 0.f;
        }
#pragma unroll
        for (int c8 = 0; c8 < kGuChunks; ++c8) {
            const int c = c8 * 256 + lane * 8;
            if (c < H) {
#pragma unroll
                for (int i = 0; i < MAXP; ++i) {
                    if (i < np) {
                        const uint4 xv = ld_cached16(a.x + (size_t)m.tok[qb + i] * H + c);
                        ag[i] = dot8(wg[c8], xv, ag[i]);
                        au[i] = dot8(wu[c8], xv, au[i]);
                    }
                }
            }
        }
#pragma unroll
        for (int i = 0; i < MAXP; ++i) {
            if (i < np) {
                const float g = round_bf16(warp_sum(ag[i]));
                const float v = round_bf16(warp_sum(au[i]));
                if (lane == i) {
                    const float s = g / (1.0f + expf(-g));
                    a.act[(size_t)m.pair[qb + i] * I + j] = __float2bfloat16_rn(s * v);
                }
            }
        }
    }
}

// Units k = (u - u_lo) * I + j for u in [u_lo, m.nu); this warp takes
// k = wid, wid + nw, ...; returns false if the kernel is aborting.
template <int MAXP>
__device__ bool gateup_units(const GroupCompute &a, const Meta &m, int u_lo, int wid, int nw, int lane,
                             const ForwardParams &fp) {
    const int I = a.I;
    const long total = (long)(m.nu - u_lo) * I;
    auto ready = [&](int u) -> bool {
        if (m.gen[u] == 0) return true;
        int ok = 1;
        if (lane == 0) ok = wait_slot(fp.slot_ready, m.slot[u], (uint32_t)m.gen[u], fp.bar, fp.wait_ns);
        return __shfl_sync(0xffffffffu, ok, 0) != 0;
    };
    uint4 wgA[kGuChunks], wuA[kGuChunks], wgB[kGuChunks], wuB[kGuChunks];
    long k = wid;
    if (k >= total) return true;
    int uA = u_lo + (int)(k / I), jA = (int)(k % I);
    if (!ready(uA)) return false;
    gu_load(a, m.slot[uA], jA, lane, wgA, wuA);
    while (true) {
        long kn = k + nw;
        int uB = 0, jB = 0;
        if (kn < total) {
            uB = u_lo + (int)(kn / I);
            jB = (int)(kn % I);
            if (!ready(uB)) return false;
            gu_load(a, m.slot[uB], jB, lane, wgB, wuB);
        }
        gu_compute<MAXP>(a, m, uA, jA, lane, wgA, wuA);
        if (kn >= total) return true;
        k = kn;
        kn = k + nw;
        if (kn < total) {
            uA = u_lo + (int)(kn / I);
            jA = (int)(kn % I);
            if (!ready(uA)) return false;
            gu_load(a, m.slot[uA], jA, lane, wgA, wuA);
        }
        gu_compute<MAXP>(a, m, uB, jB, lane, wgB, wuB);
        if (kn >= total) return true;
        k = kn;
    }
}

// ---- pipelined down x weight (decode sizes) --------------------------------------
__device__ __forceinline__ void dq_load(const GroupCompute &a, int slot, int h0, int lane,
                                        uint4 (&wv)[4][kDqChunks]) {
    const int H = a.H, I = a.I;
    const int nr = min(4, H - h0);
    const __nv_bfloat16 *wbase = a.w2 + (size_t)slot * (size_t)H * I + (size_t)h0 * I;
#pragma unroll
    for (int c4 = 0; c4 < kDqChunks; ++c4) {
        const int c = c4 * 256 + lane * 8;
        if (c < I) {
#pragma unroll
            for (int r = 0; r < 4; ++r) wv[r][c4] = ld_cg16(wbase + (size_t)(r < nr ? r : 0) * I + c);
        }
    }
}

template <int MAXQ>
__device__ __forceinline__ void dq_compute(const GroupCompute &a, const Meta &m, int u, int h0,
                                           int lane, const uint4 (&wv)[4][kDqChunks]) {
    const int H = a.H, I = a.I;
    const int nr = min(4, H - h0);
    const int q0 = m.off[u], q1 = m.off[u + 1];
    for (int qb = q0; qb < q1; qb += MAXQ) {
        const int np = min(MAXQ, q1 - qb);
        float acc[4][MAXQ];
#pragma unroll
        for (int i = 0; i < MAXQ; ++i)
#pragma unroll
            for (int r = 0; r < 4; ++r) acc[r][i] = 0.f;
#pragma unroll
        for (int c4 = 0; c4 < kDqChunks; ++c4) {
            const int c = c4 * 256 + lane * 8;
            if (c < I) {
#pragma unroll
                for (int i = 0; i < MAXQ; ++i) {
                    if (i < np) {
                        const uint4 av = ld_cg16(a.act + (size_t)m.pair[qb + i] * I + c);
#pragma unroll
                        for (int r = 0; r < 4; ++r) acc[r][i] = dot8(wv[r][c4], av, acc[r][i]);
                    }
                }
            }
        }
#pragma unroll
        for (int i = 0; i < MAXQ; ++i) {
            if (i < np) {
                const int p = m.pair[qb + i];
                const float wp = a.topk_w[p];
#pragma unroll
                for (int r = 0; r < 4; ++r) {
                    const float s = warp_sum(acc[r][i]);
                    if (lane == 0 && r < nr) a.y[(size_t)p * H + h0 + r] = __float2bfloat16_rn(s * wp);
                }
            }
        }
    }
}

// The last of the nu units of row quad q to finish sums the group's tokens.
__device__ __forceinline__ void quad_arrive(const GroupCompute &a, int q, int nu, int lane) {
    __threadfence();
    __syncwarp();
    int last = 0;
    if (lane == 0) last = (atomicAdd(&a.counters[q], 1) == nu - 1);
    if (__shfl_sync(0xffffffffu, last, 0)) {
        __threadfence();
        combine_rows(a, q * 4, 4, lane, 32);
        if (lane == 0) a.counters[q] = 0;
    }
}

template <int MAXQ>
__device__ void down_units(const GroupCompute &a, const Meta &m, int wid, int nw, int lane) {
    const int nq = (a.H + 3) / 4;
    const long total = (long)m.nu * nq;
    uint4 A[4][kDqChunks];
    for (long k = wid; k < total; k += nw) {
        const int u = (int)(k / nq), q = (int)(k % nq);
        dq_load(a, m.slot[u], q * 4, lane, A);
        dq_compute<MAXQ>(a, m, u, q * 4, lane, A);
        quad_arrive(a, q, m.nu, lane);
    }
}

// Generic (non-pipelined) bodies for groups beyond the shared-memory lists.
template <int MAXP>
__device__ __forceinline__ void gateup_generic(const GroupCompute &gc, const int32_t *ugen, int u_lo, int nu,
                                            int wid, int nw, int lane, const ForwardParams &a) {
    const int I = gc.I;
    const int n1 = (nu - u_lo) * I;
    for (int unit = wid; unit < n1; unit += nw) {
        const int u = u_lo + unit / I, j = unit % I;
        const uint32_t need = ugen ? (uint32_t)__ldcg(ugen + u) : 0u;
        if (need != 0) {
            int ok = 1;
            if (lane == 0) ok = wait_slot(a.slot_ready, __ldcg(gc.u_slot + u), need, a.bar, a.wait_ns);
            if (!__shfl_sync(0xffffffffu, ok, 0)) return;
        }
        gateup_rowpair<MAXP, true>(gc, u, j, lane);
    }
}

template <int MAXQ>
__device__ __forceinline__ void down_generic(const GroupCompute &gc, int nu, int wid, int nw, int lane) {
    const int nq = (gc.H + 3) / 4;
    const int n2 = nu * nq;
    for (int unit = wid; unit < n2; unit += nw) {
        const int u = unit / nq, q = unit - u * nq;
        down_quad<MAXQ, true>(gc, u, q * 4, lane);
        quad_arrive(gc, q, nu, lane);
    }
}

// Block-local lists of the experts resident before the call (speculative
// phase 1).  Returns false when speculation does not apply (more experts than
// the cap: several groups; or ids out of range: the pager reports them).
// `pos` is scratch for E ints.
__device__ bool build_spec_meta(const ForwardParams &fp, Meta &m, int *pos) {
    __shared__ uint32_t s_mask[32];
    __shared__ int s_flag;
    __shared__ int s_fill[kMetaU];
    const PagerParams &pg = fp.pg;
    const int P = pg.T * pg.K, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    if (P > kSpecMaxPairs || pg.E > 1024) return false;
    if (tid < 32) s_mask[tid] = 0;
    if (tid == 0) s_flag = 0;
    __syncthreads();
    for (int p = tid; p < P; p += blockDim.x) {
        const long long e = load_id64(pg.ids, pg.ids64, p);
        if (e < 0 || e >= pg.E) {
            s_flag = 1;
        } else {
            atomicOr(&s_mask[e >> 5], 1u << (e & 31));
            m.pair[p] = (int)e;  // expert of pair p, for now
        }
    }
    __syncthreads();
    if (warp == 0) {
        const uint32_t w = s_mask[lane];
        const int total = __reduce_add_sync(0xffffffffu, __popc(w));
        // pre-call residents, ascending, with their slots (block 0 writes the
        // new map back only after the first grid barrier)
        uint32_t keep = 0;
        for (uint32_t v = w; v;) {
            const int b = __ffs(v) - 1;
            v &= v - 1;
            if (pg.emap[lane * 32 + b] >= 0) keep |= 1u << b;
        }
        const int c = __popc(keep);
        int incl = c;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int v = __shfl_up_sync(0xffffffffu, incl, o);
            if (lane >= o) incl += v;
        }
        int idx = incl - c;
        for (uint32_t v = keep; v;) {
            const int b = __ffs(v) - 1;
            v &= v - 1;
            const int e = lane * 32 + b;
            m.slot[idx] = pg.emap[e];
            m.gen[idx] = 0;
            pos[e] = idx;
            ++idx;
        }
        for (uint32_t v = w & ~keep; v;) {
            const int b = __ffs(v) - 1;
            v &= v - 1;
            pos[lane * 32 + b] = -1;
        }
        const int nres = __shfl_sync(0xffffffffu, incl, 31);
        if (lane == 0) {
            m.nu = nres;
            if (total > pg.cap) s_flag = 1;
        }
    }
    __syncthreads();
    if (s_flag) return false;
    const int nu = m.nu;
    // pairs of each resident expert (CSR; pair order within an expert is free)
    for (int i = tid; i <= nu; i += blockDim.x) m.off[i] = 0;
    for (int i = tid; i < nu; i += blockDim.x) s_fill[i] = 0;
    __syncthreads();
    const int p = tid;  // P <= kSpecMaxPairs == blockDim.x
    const int my_i = p < P ? pos[m.pair[p]] : -1;
    if (my_i >= 0) atomicAdd(&m.off[my_i + 1], 1);
    __syncthreads();
    if (tid == 0) {
        int maxnp = 0;
        for (int i = 1; i <= nu; ++i) {
            maxnp = max(maxnp, m.off[i]);
            m.off[i] += m.off[i - 1];
        }
        m.maxnp = maxnp;
    }
    __syncthreads();
    const int at = my_i >= 0 ? m.off[my_i] + atomicAdd(&s_fill[my_i], 1) : -1;
    __syncthreads();  // every m.pair[] (expert ids) is read before it is overwritten
    if (at >= 0) {
        m.pair[at] = p;
        m.tok[at] = p / pg.K;
    }
    __syncthreads();
    return true;
}

// Group g's lists from the pager's device output into shared memory.
__device__ bool load_meta(const ForwardParams &fp, int g, long p0, int nu, int np_total, Meta &m) {
    if (nu > kMetaU || np_total > kMetaP) return false;
    const PagerParams &pg = fp.pg;
    const int tid = threadIdx.x;
    for (int i = tid; i < nu; i += blockDim.x) {
        m.slot[i] = __ldcg(pg.u_slot + p0 + i);
        m.gen[i] = __ldcg(pg.u_gen + p0 + i);
    }
    for (int i = tid; i <= nu; i += blockDim.x) m.off[i] = __ldcg(pg.u_off + p0 + g + i);
    for (int i = tid; i < np_total; i += blockDim.x) {
        const int p = __ldcg(pg.u_pairs + p0 + i);
        m.pair[i] = p;
        m.tok[i] = p / pg.K;
    }
    __syncthreads();
    if (tid == 0) {
        int maxnp = 0;
        for (int i = 0; i < nu; ++i) maxnp = max(maxnp, m.off[i + 1] - m.off[i]);
        m.maxnp = maxnp;
        m.nu = nu;
    }
    __syncthreads();
    return true;
}

// FAST: decode sizes (every group's lists fit in shared memory, H <= 2048,
// I <= 1024): speculative start and pipelined units.  Otherwise the generic
// bodies.  The host picks the variant from the shapes alone.
template <int MAXP, bool FAST>
__global__ void __launch_bounds__(kFwdThreads, kBlocksPerSm) forward_kernel(const __grid_constant__ ForwardParams a) {
    extern __shared__ __align__(16) unsigned char smem[];
    __shared__ Meta meta;
    constexpr int MAXQ = MAXP < 4 ? MAXP : 4;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, tid = threadIdx.x;
    const int nwarps = gridDim.x * kWarpsPerBlock;
    const int gw = blockIdx.x * kWarpsPerBlock + warp;
    const PagerParams &pg = a.pg;
    unsigned long long *tr = a.trace;
#define WISP_TRACE(slot)                                                                 \
    do {                                                                                 \
        if (tr && tid == 0) tr[8 + blockIdx.x * 4 + (slot)] = globaltimer_ns();          \
    } while (0)
#define WISP_TRACE0(slot)                                                                \
    do {                                                                                 \
        if (tr && tid == 0 && blockIdx.x == 0) tr[(slot)] = globaltimer_ns();            \
    } while (0)
    WISP_TRACE(0);
    WISP_TRACE0(0);

    // ---- phase 0: pager on block 0, speculative gate-up on the others --------------
    if (blockIdx.x == 0) {
        pager_body(pg, smem);
        WISP_TRACE0(1);
    } else if (FAST && build_spec_meta(a, meta, reinterpret_cast<int *>(smem))) {
        GroupCompute gc = a.gc;
        gc.t0 = 0;
        gc.t1 = pg.T;
        gateup_units<MAXP>(gc, meta, 0, gw - kWarpsPerBlock, nwarps - kWarpsPerBlock, lane, a);
        WISP_TRACE(1);
    }
    if (!grid_barrier(a.bar, a.wait_ns)) goto done;
    WISP_TRACE0(2);
    if (blockIdx.x == 0) pager_finish(pg, smem, a.publish != 0);
    {
        const int status = __ldcg(pg.dev_hdr + kHdrStatus);
        if (status != WISP_OK) {
            if (blockIdx.x == 0 && tid == 0) set_status(a.bar, status);
            goto done;
        }
        const int G = __ldcg(pg.dev_hdr + kHdrGroups);
        const int K = a.gc.K, H = a.gc.H, I = a.gc.I;
        const int P = pg.T * pg.K;
        // mirrors build_spec_meta's condition: one group <=> the experts fit the cap
        const bool spec_ran = FAST && (G == 1) && (P <= kSpecMaxPairs) && (gridDim.x > 1) && pg.E <= 1024;
        for (int g = 0; g < G; ++g) {
            GroupCompute gc = a.gc;
            const int t0 = __ldcg(pg.grp_start + g), t1 = __ldcg(pg.grp_start + g + 1);
            const long p0 = (long)t0 * K;
            const int nu = __ldcg(pg.grp_nu + g);
            const int u_lo = (g == 0 && spec_ran) ? __ldcg(pg.grp_nhit + 0) : 0;
            gc.t0 = t0;
            gc.t1 = t1;
            if (FAST) load_meta(a, g, p0, nu, (t1 - t0) * K, meta);
            // phase 1: gate-up + SiLU-mul
            if (FAST) {
                gateup_units<MAXP>(gc, meta, u_lo, gw, nwarps, lane, a);
            } else {
                gc.u_slot = pg.u_slot + p0;
                gc.u_off = pg.u_off + p0 + g;
                gc.u_pairs = pg.u_pairs + p0;
                gateup_generic<MAXP>(gc, pg.u_gen + p0, u_lo, nu, gw, nwarps, lane, a);
            }
            __syncthreads();
            WISP_TRACE(2);
            if (!grid_barrier(a.bar, a.wait_ns)) goto done;
            WISP_TRACE0(3);
            // phase 2: down x weight, last arrival per row quad combines
            if (FAST) {
                down_units<MAXQ>(gc, meta, gw, nwarps, lane);
            } else {
                gc.u_slot = pg.u_slot + p0;
                gc.u_off = pg.u_off + p0 + g;
                gc.u_pairs = pg.u_pairs + p0;
                down_generic<MAXQ>(gc, nu, gw, nwarps, lane);
            }
            __syncthreads();
            WISP_TRACE(3);
            if (g + 1 < G) {
                // later groups may page into slots this group read: publish "done"
                if (!grid_barrier(a.bar, a.wait_ns)) goto done;
                if (blockIdx.x == 0 && tid == 0) {
                    *reinterpret_cast<volatile unsigned long long *>(a.done_word) =
                        ((unsigned long long)pg.seq << 32) | (unsigned)(g + 1);
                    __threadfence_system();
                }
            }
        }
    }
done:
    WISP_TRACE0(4);
#undef WISP_TRACE
#undef WISP_TRACE0
    if (blockIdx.x == 0 && tid == 0) {
        const unsigned int st = *reinterpret_cast<volatile unsigned int *>(a.bar + kBarStatus);
        if (st != 0) {
            *a.status_word = (int)st;  // sticky, cleared by the host
            __threadfence_system();
        }
    }
}

template <int MAXP, bool FAST>
int launch_t(const ForwardParams &p, size_t smem, cudaStream_t stream) {
    static int nblk_per_sm[64];
    static size_t smem_set[64];
    int dev = 0;
    WISP_CUDA_TRY(cudaGetDevice(&dev));
    if (dev < 0 || dev >= 64) return WISP_ERR_INVALID;
    if (smem_set[dev] < smem || !nblk_per_sm[dev]) {
        WISP_CUDA_TRY(cudaFuncSetAttribute(forward_kernel<MAXP, FAST>,
                                           cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
        int nb = 0;
        WISP_CUDA_TRY(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&nb, forward_kernel<MAXP, FAST>, kFwdThreads, smem));
        if (nb < 1) return set_error("forward kernel does not fit on an SM"), WISP_ERR_UNSUPPORTED;
        nblk_per_sm[dev] = nb > kBlocksPerSm ? kBlocksPerSm : nb;
        smem_set[dev] = smem;
    }
    int sms = 0;
    WISP_CUDA_TRY(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
    dim3 grid(sms * nblk_per_sm[dev]), block(kFwdThreads);
    ForwardParams arg = p;
    void *args[] = {&arg};
    WISP_CUDA_TRY(cudaLaunchCooperativeKernel((const void *)forward_kernel<MAXP, FAST>, grid, block, args,
                                              smem, stream));
    return WISP_OK;
}

}  // namespace

int launch_forward(const ForwardParams &p, int max_tokens_per_group, cudaStream_t stream) {
    size_t smem = pager_smem_bytes(p.pg.E, p.pg.cap, p.pg.T, p.pg.K);
    smem = smem > sizeof(int) * 1024 ? smem : sizeof(int) * 1024;  // speculation's expert index
    const bool fast = (long)p.pg.T * p.pg.K <= kMetaP && p.gc.H <= kGuChunks * 256 &&
                      p.gc.I <= kDqChunks * 256;
    if (fast) {
        if (max_tokens_per_group <= 1) return launch_t<1, true>(p, smem, stream);
        if (max_tokens_per_group <= 2) return launch_t<2, true>(p, smem, stream);
        if (max_tokens_per_group <= 4) return launch_t<4, true>(p, smem, stream);
        return launch_t<8, true>(p, smem, stream);  // more pairs per expert: further passes
    }
    if (max_tokens_per_group <= 1) return launch_t<1, false>(p, smem, stream);
    if (max_tokens_per_group <= 4) return launch_t<4, false>(p, smem, stream);
    return launch_t<8, false>(p, smem, stream);
}

}  // namespace wisp
