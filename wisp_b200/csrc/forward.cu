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

// ---- TMA-fed units (decode sizes) --------------------------------------------
// Each warp owns kStages shared-memory buffers of kStageBytes with one
// mbarrier each.  Lane 0 streams a unit's weight rows (contiguous blocks) in
// with cp.async.bulk; the warp computes from shared memory while the copies of
// its next units are in flight.  Every mbarrier wait is bounded in time.
constexpr int kStages = 2;
constexpr int kStageBytes = 8192;  // >= 2 rows x H (gate-up) and 4 rows x I (down), bf16
constexpr int kPubLane = 31;       // lane that stores and publishes gate-up rows

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return (uint32_t)__cvta_generic_to_shared(p);
}
__device__ __forceinline__ void mbar_init(uint64_t *bar, int count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}
__device__ __forceinline__ void fence_proxy_async() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Per-warp copy pipeline state.
struct WarpPipe {
    unsigned char *buf;  // kStages * kStageBytes
    uint64_t *bar;       // kStages mbarriers
    uint32_t phase;      // bit s: parity to wait for on stage s
    uint32_t pending;    // bit s: a copy into stage s has not been waited for
};

// Wait for stage s (bounded); on timeout record it and abort.
__device__ bool pipe_wait(WarpPipe &w, int s, const ForwardParams &fp) {
    const uint32_t par = (w.phase >> s) & 1u;
    if (!mbar_try_wait(w.bar + s, par)) {
        const unsigned long long t0 = globaltimer_ns();
        while (!mbar_try_wait(w.bar + s, par)) {
            if ((long long)(globaltimer_ns() - t0) > fp.wait_ns) {
                set_status(fp.bar, WISP_ERR_TIMEOUT);
                atomicExch(fp.bar + kBarAbort, 1u);
                return false;
            }
        }
    }
    w.phase ^= 1u << s;
    w.pending &= ~(1u << s);
    return true;
}

// Before leaving on an abort: let the copies still landing in this warp's
// buffers finish (each wait bounded), so no copy outlives the block.
__device__ void pipe_drain(WarpPipe &w, const ForwardParams &fp) {
    for (int s = 0; s < kStages; ++s) {
        if (!((w.pending >> s) & 1u)) continue;
        const uint32_t par = (w.phase >> s) & 1u;
        const unsigned long long t0 = globaltimer_ns();
        while (!mbar_try_wait(w.bar + s, par))
            if ((long long)(globaltimer_ns() - t0) > fp.wait_ns) break;
        w.phase ^= 1u << s;
    }
    w.pending = 0;
}

// Lane 0 (the caller has established the slot is ready): copy `n` blocks.
__device__ __forceinline__ void pipe_issue(WarpPipe &w, int s, const void *src0, uint32_t b0,
                                           const void *src1, uint32_t b1) {
    unsigned char *dst = w.buf + s * kStageBytes;
    fence_proxy_async();
    mbar_expect_tx(w.bar + s, b0 + b1);
    bulk_g2s(dst, src0, b0, w.bar + s);
    if (b1) bulk_g2s(dst + b0, src1, b1, w.bar + s);
}

// Gate-up units k = (u - u_lo) * I + j, u in [u_lo, m.nu); this warp takes
// k = wid, wid + nw, ...  Returns false when the kernel is aborting.
template <int MAXP>
__device__ bool gateup_units(const GroupCompute &a, const Meta &m, int u_lo, int wid, int nw, int lane,
                             const ForwardParams &fp, WarpPipe &w, unsigned int *done1) {
    const int H = a.H, I = a.I;
    const uint32_t rowb = (uint32_t)H * 2;
    const long total = (long)(m.nu - u_lo) * I;
    auto issue = [&](long k, int s) -> bool {
        const int u = u_lo + (int)(k / I), j = (int)(k % I);
        if (m.gen[u] != 0) {  // expert paged in during this call: its slot must have landed
            int ok = 1;
            if (lane == 0) ok = wait_slot(fp.slot_ready, m.slot[u], (uint32_t)m.gen[u], fp.bar, fp.wait_ns);
            if (!__shfl_sync(0xffffffffu, ok, 0)) return false;
        }
        if (lane == 0) {
            const __nv_bfloat16 *g = a.w13 + (size_t)m.slot[u] * (size_t)(2 * I) * H + (size_t)j * H;
            pipe_issue(w, s, g, rowb, g + (size_t)I * H, rowb);
        }
        w.pending |= 1u << s;
        return true;
    };
    bool ok = true;
    for (int s = 0; s < kStages && ok; ++s) {
        const long k = wid + (long)s * nw;
        if (k < total) ok = issue(k, s);
    }
    // publication of the previous unit's rows, one unit late: by then its stores
    // have completed and the fence costs little
    // (the stores and the fence are on kPubLane, not on lane 0 which issues the
    // copies: a fence must not wait for this warp's copies in flight)
    int pub_u = -1;
    unsigned pub_n = 0;
    auto publish = [&]() {
        if (done1 && pub_n && lane == kPubLane) {
            __threadfence();
            atomicAdd(done1 + pub_u, pub_n);
        }
        pub_n = 0;
    };
    long i = 0;
    for (long k = wid; ok && k < total; k += nw, ++i) {
        const int s = (int)(i % kStages);
        if (!pipe_wait(w, s, fp)) {
            ok = false;
            break;
        }
        publish();
        const int u = u_lo + (int)(k / I), j = (int)(k % I);
        const uint4 *gs = reinterpret_cast<const uint4 *>(w.buf + s * kStageBytes);
        const uint4 *us = reinterpret_cast<const uint4 *>(w.buf + s * kStageBytes + rowb);
        const int q0 = m.off[u], q1 = m.off[u + 1];
        for (int qb = q0; qb < q1; qb += MAXP) {
            const int np = min(MAXP, q1 - qb);
            float ag[MAXP], au[MAXP];
#pragma unroll
            for (int t = 0; t < MAXP; ++t) {
                ag[t] = 0.f;
                au[t] = 0.f;
            }
#pragma unroll
            for (int c8 = 0; c8 < kGuChunks; ++c8) {
                const int c = c8 * 256 + lane * 8;
                if (c < H) {
                    const uint4 wg = gs[c >> 3], wu = us[c >> 3];
#pragma unroll
                    for (int t = 0; t < MAXP; ++t) {
                        if (t < np) {
                            const uint4 xv = ld_cached16(a.x + (size_t)m.tok[qb + t] * H + c);
                            ag[t] = dot8(wg, xv, ag[t]);
                            au[t] = dot8(wu, xv, au[t]);
                        }
                    }
                }
            }
#pragma unroll
            for (int t = 0; t < MAXP; ++t) {
                if (t < np) {
                    const float g = round_bf16(warp_sum(ag[t]));
                    const float v = round_bf16(warp_sum(au[t]));
                    if (lane == kPubLane) {  // one lane stores every pair's row j and publishes them
                        const float sg = g / (1.0f + expf(-g));
                        a.act[(size_t)m.pair[qb + t] * I + j] = __float2bfloat16_rn(sg * v);
                    }
                }
            }
        }
        pub_u = u;
        pub_n = (unsigned)(q1 - q0);
        __syncwarp();
        const long kn = k + (long)kStages * nw;
        if (kn < total) ok = issue(kn, s);
    }
    if (!ok) {
        pipe_drain(w, fp);
        return false;
    }
    publish();
    return true;
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

// Wait (lane 0, bounded) until every gate-up row of expert u is published.
__device__ bool wait_act(const unsigned int *done1, int u, unsigned int need, const ForwardParams &fp,
                         int lane) {
    int ok = 1;
    if (lane == 0) {
        volatile const unsigned int *f = done1 + u;
        if (*f < need) {
            volatile unsigned int *vabort = fp.bar + kBarAbort;
            const unsigned long long t0 = globaltimer_ns();
            while (*f < need) {
                if (*vabort) {
                    ok = 0;
                    break;
                }
                if ((long long)(globaltimer_ns() - t0) > fp.wait_ns) {
                    set_status(fp.bar, WISP_ERR_TIMEOUT);
                    atomicExch(fp.bar + kBarAbort, 1u);
                    ok = 0;
                    break;
                }
                __nanosleep(64);
            }
        }
        __threadfence();
    }
    return __shfl_sync(0xffffffffu, ok, 0) != 0;
}

// Down units k = u * nq + q (four rows h0 = 4q.. of expert u, one contiguous
// block of W2) for u < m.nu.  Units go out in chunks of kDownChunk
// consecutive units (mostly one expert, whose activation rows then stay in
// registers), chunks round-robin over the warps.  With `done1`, a unit first
// waits until its expert's activations are complete (its W2 copy is already
// in flight).  The weighted y of every unit goes to global memory; at the end
// the warp fences once and its lanes arrive on the row quads' counters in
// parallel; the last arrival of a quad sums the group's tokens over k in
// routing order for those rows.
constexpr int kDownChunk = 4;
template <int MAXQ>
__device__ bool down_units(const GroupCompute &a, const Meta &m, int wid, int nw, int lane,
                           const ForwardParams &fp, WarpPipe &w, const unsigned int *done1) {
    const int H = a.H, I = a.I;
    const int nq = (H + 3) / 4;
    const long total = (long)m.nu * nq;
    // the i-th unit of this warp (may be >= total past the last one)
    auto unit_of = [&](long i) -> long {
        return ((long)wid + (i / kDownChunk) * nw) * kDownChunk + (i % kDownChunk);
    };
    long count = 0;
    while (unit_of(count) < total) ++count;  // at most a few chunks per warp
    if (count == 0) return true;
    // a unit of an expert paged in during this call reads its slot only after
    // the page-in has landed
    auto issue = [&](long i, int s) -> bool {
        const long k = unit_of(i);
        const int u = (int)(k / nq), q = (int)(k % nq);
        const int nr = min(4, H - 4 * q);
        if (m.gen[u] != 0) {
            int rdy = 1;
            if (lane == 0) rdy = wait_slot(fp.slot_ready, m.slot[u], (uint32_t)m.gen[u], fp.bar, fp.wait_ns);
            if (!__shfl_sync(0xffffffffu, rdy, 0)) return false;
        }
        if (lane == 0)
            pipe_issue(w, s, a.w2 + (size_t)m.slot[u] * (size_t)H * I + (size_t)(4 * q) * I,
                       (uint32_t)nr * I * 2, nullptr, 0);
        w.pending |= 1u << s;
        return true;
    };
    bool ok = true;
    for (int s = 0; s < kStages && ok; ++s)
        if (s < count) ok = issue(s, s);
    uint4 act[MAXQ][kDqChunks];
    int act_u = -1;
    for (long i = 0; ok && i < count; ++i) {
        const int s = (int)(i % kStages);
        const long k = unit_of(i);
        const int u = (int)(k / nq), q = (int)(k % nq), h0 = 4 * q;
        const int q0 = m.off[u], q1 = m.off[u + 1];
        if (done1 && u != act_u && !wait_act(done1, u, (unsigned)(I * (q1 - q0)), fp, lane)) {
            ok = false;
            break;
        }
        const bool cached = (q1 - q0) <= MAXQ;
        if (cached && u != act_u) {  // this expert's activation rows, reused by its next quads
#pragma unroll
            for (int t = 0; t < MAXQ; ++t)
                if (t < q1 - q0)
#pragma unroll
                    for (int c4 = 0; c4 < kDqChunks; ++c4) {
                        const int c = c4 * 256 + lane * 8;
                        if (c < I) act[t][c4] = ld_cg16(a.act + (size_t)m.pair[q0 + t] * I + c);
                    }
        }
        act_u = u;
        if (!pipe_wait(w, s, fp)) {
            ok = false;
            break;
        }
        const int nr = min(4, H - h0);
        const uint4 *ws = reinterpret_cast<const uint4 *>(w.buf + s * kStageBytes);
        for (int qb = q0; qb < q1; qb += MAXQ) {
            const int np = min(MAXQ, q1 - qb);
            float acc[4][MAXQ];
#pragma unroll
            for (int t = 0; t < MAXQ; ++t)
#pragma unroll
                for (int r = 0; r < 4; ++r) acc[r][t] = 0.f;
#pragma unroll
            for (int c4 = 0; c4 < kDqChunks; ++c4) {
                const int c = c4 * 256 + lane * 8;
                if (c < I) {
                    uint4 wv[4];
#pragma unroll
                    for (int r = 0; r < 4; ++r) wv[r] = ws[((r < nr ? r : 0) * I + c) >> 3];
#pragma unroll
                    for (int t = 0; t < MAXQ; ++t) {
                        if (t < np) {
                            const uint4 av =
                                cached ? act[t][c4] : ld_cg16(a.act + (size_t)m.pair[qb + t] * I + c);
#pragma unroll
                            for (int r = 0; r < 4; ++r) acc[r][t] = dot8(wv[r], av, acc[r][t]);
                        }
                    }
                }
            }
#pragma unroll
            for (int t = 0; t < MAXQ; ++t) {
                if (t < np) {
                    const int p = m.pair[qb + t];
                    const float wp = a.topk_w[p];
#pragma unroll
                    for (int r = 0; r < 4; ++r) {
                        const float sum = warp_sum(acc[r][t]);
                        if (lane == r && r < nr) a.y[(size_t)p * H + h0 + r] = __float2bfloat16_rn(sum * wp);
                    }
                }
            }
        }
        __syncwarp();
        if (i + kStages < count) ok = issue(i + kStages, s);
    }
    if (!ok) {
        pipe_drain(w, fp);
        return false;
    }
    // arrivals: one fence, then one lane per unit
    __threadfence();
    __syncwarp();
    for (long ib = 0; ib < count; ib += 32) {
        const long i = ib + lane;
        int last = 0, q = 0;
        if (i < count) {
            q = (int)(unit_of(i) % nq);
            last = (atomicAdd(&a.counters[q], 1) == m.nu - 1);
        }
        unsigned todo = __ballot_sync(0xffffffffu, last);
        if (todo) __threadfence();
        while (todo) {
            const int l = __ffs(todo) - 1;
            todo &= todo - 1;
            const int ql = __shfl_sync(0xffffffffu, q, l);
            combine_rows(a, ql * 4, 4, lane, 32);
            if (lane == 0) a.counters[ql] = 0;
        }
    }
    return true;
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

// Bounded wait (thread 0 of the block) until *word reaches `want`; then every
// thread of the block sees the words written before it.
__device__ bool block_wait_word(const unsigned int *word, unsigned int want, const ForwardParams &fp,
                                bool equal) {
    __shared__ int s_ok;
    if (threadIdx.x == 0) {
        int ok = 1;
        volatile const unsigned int *f = word;
        volatile unsigned int *vabort = fp.bar + kBarAbort;
        const unsigned long long t0 = globaltimer_ns();
        while (equal ? (*f != want) : (*f < want)) {
            if (*vabort) {
                ok = 0;
                break;
            }
            if ((long long)(globaltimer_ns() - t0) > fp.wait_ns) {
                set_status(fp.bar, WISP_ERR_TIMEOUT);
                atomicExch(fp.bar + kBarAbort, 1u);
                ok = 0;
                break;
            }
            __nanosleep(32);
        }
        __threadfence();
        s_ok = ok;
    }
    __syncthreads();
    return s_ok != 0;
}

// FAST: decode sizes (every group's lists fit in shared memory, H <= 2048,
// I <= 1024): TMA-fed warp units, a speculative start, and for a call that
// forms one token group no grid barrier at all (dataflow counters).
// Otherwise the generic bodies with grid barriers between phases.  The host
// picks the variant from the shapes alone.
template <int MAXP, bool FAST>
__global__ void __launch_bounds__(kFwdThreads, kBlocksPerSm) forward_kernel(const __grid_constant__ ForwardParams a) {
    extern __shared__ __align__(16) unsigned char smem[];
    __shared__ Meta meta;
    constexpr int MAXQ = MAXP < 4 ? MAXP : 4;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, tid = threadIdx.x;
    const int nwarps = gridDim.x * kWarpsPerBlock;
    const int gw = blockIdx.x * kWarpsPerBlock + warp;
    const PagerParams &pg = a.pg;
    unsigned int *done1 = a.flow + kFlowDone1 + a.epoch * kFlowMaxU;
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

    // per-warp copy pipelines (FAST variant); buffers overlay the pager's shared
    // memory, which block 0 is done with before its first copy
    __shared__ __align__(8) uint64_t s_bars[kWarpsPerBlock][kStages];
    WarpPipe pipe{};
    if (FAST) {
        pipe.buf = smem + (size_t)warp * kStages * kStageBytes;
        pipe.bar = s_bars[warp];
        if (lane == 0) {
            for (int st = 0; st < kStages; ++st) mbar_init(pipe.bar + st, 1);
            fence_proxy_async();
        }
        __syncwarp();
    }

    // ---- phase 0 ------------------------------------------------------------------
    // block 0: pager, publish its outputs, wait until no block still reads the
    // pre-call expert map, write the new state back.  Other blocks: read the
    // pre-call map (speculation lists), say so, run gate-up for the experts
    // that were resident before the call.
    bool spec_here = false;
    if (blockIdx.x == 0) {
        if (tid == 0) {  // the counters the next launch uses start at zero
            a.flow[kFlowSpecRead + (a.epoch ^ 1)] = 0;
        }
        for (int i = tid; i < kFlowMaxU; i += kFwdThreads)
            a.flow[kFlowDone1 + (a.epoch ^ 1) * kFlowMaxU + i] = 0;
        pager_body(pg, smem);
        if (tid == 0) {
            __threadfence();
            *reinterpret_cast<volatile unsigned int *>(a.flow + kFlowPagerDone) = pg.seq;
        }
        WISP_TRACE0(1);
        if (!block_wait_word(a.flow + kFlowSpecRead + a.epoch, gridDim.x - 1, a, false)) goto done;
        pager_finish(pg, smem, a.publish != 0);
        WISP_TRACE0(2);
    } else {
        if (FAST) spec_here = build_spec_meta(a, meta, reinterpret_cast<int *>(smem));
        __syncthreads();
        if (tid == 0) {
            __threadfence();
            atomicAdd(a.flow + kFlowSpecRead + a.epoch, 1u);
        }
        if (spec_here) {
            GroupCompute gc = a.gc;
            gc.t0 = 0;
            gc.t1 = pg.T;
            gateup_units<MAXP>(gc, meta, 0, gw - kWarpsPerBlock, nwarps - kWarpsPerBlock, lane, a, pipe,
                               done1);
        }
        __syncthreads();
        WISP_TRACE(1);
        if (!block_wait_word(a.flow + kFlowPagerDone, pg.seq, a, true)) goto done;
    }
    {
        const int status = __ldcg(pg.dev_hdr + kHdrStatus);
        if (status != WISP_OK) {
            if (blockIdx.x == 0 && tid == 0) set_status(a.bar, status);
            goto done;
        }
        const int G = __ldcg(pg.dev_hdr + kHdrGroups);
        const int K = a.gc.K;
        const int P = pg.T * pg.K;
        // mirrors build_spec_meta's condition: one group <=> the experts fit the cap
        const bool spec_ran = FAST && (G == 1) && (P <= kSpecMaxPairs) && (gridDim.x > 1) && pg.E <= 1024;
        if (FAST && G == 1) {
            // ---- one group: dataflow, no grid barrier -------------------------------------
            GroupCompute gc = a.gc;
            const int t1 = __ldcg(pg.grp_start + 1);
            const int nu = __ldcg(pg.grp_nu + 0);
            const int u_lo = spec_ran ? __ldcg(pg.grp_nhit + 0) : 0;
            gc.t0 = 0;
            gc.t1 = t1;
            load_meta(a, 0, 0, nu, t1 * K, meta);
            if (!gateup_units<MAXP>(gc, meta, u_lo, gw, nwarps, lane, a, pipe, done1)) goto done;
            __syncthreads();
            WISP_TRACE(2);
            down_units<MAXQ>(gc, meta, gw, nwarps, lane, a, pipe, done1);
            __syncthreads();
            WISP_TRACE(3);
        } else {
            // ---- several groups (or the generic variant): grid barriers between phases ---------
            if (!grid_barrier(a.bar, a.wait_ns)) goto done;
            const int H = a.gc.H, I = a.gc.I;
            for (int g = 0; g < G; ++g) {
                GroupCompute gc = a.gc;
                const int t0 = __ldcg(pg.grp_start + g), t1 = __ldcg(pg.grp_start + g + 1);
                const long p0 = (long)t0 * K;
                const int nu = __ldcg(pg.grp_nu + g);
                gc.t0 = t0;
                gc.t1 = t1;
                if (FAST) load_meta(a, g, p0, nu, (t1 - t0) * K, meta);
                // phase 1: gate-up + SiLU-mul
                if (FAST) {
                    gateup_units<MAXP>(gc, meta, 0, gw, nwarps, lane, a, pipe, nullptr);
                } else {
                    gc.u_slot = pg.u_slot + p0;
                    gc.u_off = pg.u_off + p0 + g;
                    gc.u_pairs = pg.u_pairs + p0;
                    gateup_generic<MAXP>(gc, pg.u_gen + p0, 0, nu, gw, nwarps, lane, a);
                }
                __syncthreads();
                WISP_TRACE(2);
                if (!grid_barrier(a.bar, a.wait_ns)) goto done;
                // phase 2: down x weight, last arrival per row quad combines
                if (FAST) {
                    down_units<MAXQ>(gc, meta, gw, nwarps, lane, a, pipe, nullptr);
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
                (void)H;
                (void)I;
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
                      p.gc.I <= kDqChunks * 256 && 2L * 2 * p.gc.H <= kStageBytes &&
                      4L * 2 * p.gc.I <= kStageBytes;
    if (fast) {
        const size_t stages = (size_t)kWarpsPerBlock * kStages * kStageBytes;
        smem = smem > stages ? smem : stages;
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
