// Persistent cooperative forward kernel: one launch per layer forward.
//
//   phase 0  block 0 runs the LRU pager (pager_body) for every token group of
//            the call.  Meanwhile, when the call's experts fit the cap (one
//            group, decode sizes), the other blocks already compute the
//            experts that were resident before the call: those are exactly
//            the pager's hits and keep their slots; block 0 writes the new
//            expert map back only after every block has read the old one;
//   units    gate-up GEMV + SiLU-mul, unit = one row pair of one unique
//            expert; down GEMV x routing weight, unit = four rows of one
//            expert.  A unit of an expert paged in during this call first
//            waits until the slot's generation flag (written by the copy
//            stream after the two copies) reaches the generation the pager
//            assigned.  The last down unit of a row quad to finish (arrival
//            counter) sums the group's tokens over k in routing order for
//            those rows.
//
// Decode sizes (FAST): each warp runs one pipelined stream of units - its
// gate-up units, then its down units - with the weight rows streamed into
// shared memory by cp.async.bulk; a down unit polls the activation rows it
// needs (each element is written once per launch over a "not written"
// pattern, so the element is its own flag: no counters or fences between the
// phases).  A call of several token groups separates the phases with grid
// barriers, and between groups block 0 publishes "group g done" to mapped
// host memory, which lets the host copy thread overwrite slots g read.  Larger
// shapes use the generic bodies of moe_body.cuh.  The arithmetic per (token,
// expert) pair is the same everywhere (moe_body.cuh documents it).
//
// Every wait (grid barrier, slot flag, copy, activation poll) is bounded by
// wait_ns of %globaltimer time; a wait that runs out sets the abort word and
// the sticky status WISP_ERR_TIMEOUT, every other wait then gives up too, and
// the kernel returns.
#include "forward.cuh"
#include "moe_body.cuh"
#include "pager_body.cuh"

namespace wisp {

namespace {

// Warps per block (block 0 runs the pager with all of them): 8 with three
// copy stages each for single-token calls (the per-warp pipeline depth
// matters most there), 12 with two stages (the same shared memory) otherwise,
// where more warps per SM hide more of each unit's latency.
constexpr int kWarpsDeep = 8;
constexpr int kWarpsWide = 12;
static_assert(kWarpsDeep * 32 >= kPagerThreads && kWarpsWide * 32 >= kPagerThreads, "the pager needs >= kPagerThreads");
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
    int total;  // speculation lists: unique experts of the call (resident or not)
    int slot[kMetaU], gen[kMetaU], off[kMetaU + 1];
    int pair[kMetaP], tok[kMetaP];
    float wt[kMetaP];  // routing weight of each list entry's pair
};

// ---- TMA-fed units (decode sizes) --------------------------------------------
// Each warp owns `nst` (2 or 3) shared-memory stages of kStageBytes with one
// mbarrier each.  Lane 0 streams a unit's weight rows (contiguous blocks) in
// with cp.async.bulk; the warp computes from shared memory while the copies of
// its next units are in flight.  Every mbarrier wait is bounded in time.
constexpr int kMaxStages = 3;
constexpr int kStageBytes = 8192;  // >= 2 rows x H (gate-up) and 4 rows x I (down), bf16
constexpr int kPubLane = 31;       // lane that stores gate-up rows
constexpr int kPairPass = 4;       // (token, k) pairs per pass over a unit's rows
constexpr int kTraceWarps = 8 + 4 * 1024;  // per-warp records (16 words) start here in the trace buffer

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
// Weight rows are read once per forward: their L2 lines go first, so the
// stream does not push the kernel's code and the small shared inputs (hidden
// states, activations, y) out of L2.
__device__ __forceinline__ uint64_t l2_evict_first_policy() {
    uint64_t pol;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
    return pol;
}
__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, uint32_t bytes, uint64_t *bar,
                                         uint64_t pol) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], "
        "%4;" ::"r"(smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(pol)
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
    unsigned char *buf;  // nst * kStageBytes
    uint64_t *bar;       // nst mbarriers
    uint32_t phase;      // bit s: parity to wait for on stage s
    uint32_t pending;    // bit s: a copy into stage s has not been waited for
    int nst;             // stages in use
    uint64_t pol;        // L2 policy of the weight copies
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
    for (int s = 0; s < w.nst; ++s) {
        if (!((w.pending >> s) & 1u)) continue;
        const uint32_t par = (w.phase >> s) & 1u;
        const unsigned long long t0 = globaltimer_ns();
        while (!mbar_try_wait(w.bar + s, par))
            if ((long long)(globaltimer_ns() - t0) > fp.wait_ns) break;
        w.phase ^= 1u << s;
    }
    w.pending = 0;
}

// Lane 0 (the caller has established the slot is ready): copy one or two blocks.
__device__ __forceinline__ void pipe_issue(WarpPipe &w, int s, const void *src0, uint32_t b0,
                                           const void *src1, uint32_t b1) {
    unsigned char *dst = w.buf + s * kStageBytes;
    fence_proxy_async();
    mbar_expect_tx(w.bar + s, b0 + b1);
    bulk_g2s(dst, src0, b0, w.bar + s, w.pol);
    if (b1) bulk_g2s(dst + b0, src1, b1, w.bar + s, w.pol);
}

// A warp's share of the units of experts [u0, u1) of the group's lists: first
// its gate-up units (unit k: expert u0 + k / I, row pair k % I; warp k % nw),
// then its down units (unit d: expert u0 + d / nq, rows 4 (d % nq) ..), dealt
// in chunks of kDownChunk consecutive units (mostly one expert, whose
// activation rows then stay in registers) round-robin over the warps,
// starting with the warp after the one that took the last gate-up unit, so
// every warp gets nearly the same number of units.  A down unit comes after
// every gate-up unit it reads in every warp's stream, so no wait can close a
// cycle.  (Releasing an expert's down units right after its last gate-up
// wave instead made warps that polled for rows still being computed hold up
// their own gate-up units; the waves convoyed.)
constexpr int kDownChunk = 4;
struct Stream {
    int u0, n_gu, n_dn, nch;  // first expert; gate-up units, down units, down chunks
    int wid, nw, I, nq;
    int nw_div, nw_mod;       // nw / I, nw % I
    int my_gu, j0;            // this warp's gate-up units; its first down chunk
};

__device__ __forceinline__ Stream make_stream(int u0, int u1, bool gu, bool dn, int wid, int nw, int I,
                                              int nq) {
    Stream s;
    const int ne = u1 > u0 ? u1 - u0 : 0;
    s.u0 = u0;
    s.n_gu = gu ? ne * I : 0;
    s.n_dn = dn ? ne * nq : 0;
    s.nch = (s.n_dn + kDownChunk - 1) / kDownChunk;
    s.wid = wid;
    s.nw = nw;
    s.I = I;
    s.nq = nq;
    s.nw_div = nw / I;
    s.nw_mod = nw - s.nw_div * I;
    s.my_gu = wid < s.n_gu ? (s.n_gu - 1 - wid) / nw + 1 : 0;
    s.j0 = (wid - s.n_gu % nw + nw) % nw;
    return s;
}

// Position in a warp's stream, advanced without divisions per item.
struct Cursor {
    int gu_left;  // gate-up items left, the current one included (0: in the down items)
    int e, r;     // current item: expert (from u0), row pair or row quad
    int j, d, d_end;
    bool done;
};

__device__ __forceinline__ void cursor_chunk(Cursor &c, const Stream &S, int j) {
    if (j >= S.nch) {
        c.done = true;
        return;
    }
    c.j = j;
    c.d = j * kDownChunk;
    c.d_end = min(c.d + kDownChunk, S.n_dn);
    c.e = c.d / S.nq;
    c.r = c.d - c.e * S.nq;
}

__device__ __forceinline__ Cursor cursor_begin(const Stream &S) {
    Cursor c;
    c.done = false;
    c.gu_left = S.my_gu;
    c.j = c.d = c.d_end = 0;
    if (c.gu_left > 0) {
        c.e = S.wid / S.I;
        c.r = S.wid - c.e * S.I;
    } else {
        c.e = c.r = 0;
        cursor_chunk(c, S, S.j0);
    }
    return c;
}

__device__ __forceinline__ void cursor_next(Cursor &c, const Stream &S) {
    if (c.gu_left > 0) {
        if (--c.gu_left > 0) {
            c.e += S.nw_div;
            c.r += S.nw_mod;
            if (c.r >= S.I) {
                c.r -= S.I;
                ++c.e;
            }
        } else {
            cursor_chunk(c, S, S.j0);
        }
        return;
    }
    if (c.done) return;
    if (++c.d < c.d_end) {
        if (++c.r == S.nq) {
            c.r = 0;
            ++c.e;
        }
    } else {
        cursor_chunk(c, S, c.j + S.nw);
    }
}

// One pass of a gate-up unit over P pairs starting at list entry qb.
template <int P>
__device__ __forceinline__ void gu_pass(const GroupCompute &a, const Meta &m, int qb, const unsigned char *st,
                                        int j, int lane) {
    const int H = a.H, I = a.I;
    const uint4 *gs = reinterpret_cast<const uint4 *>(st);
    const uint4 *us = reinterpret_cast<const uint4 *>(st + (size_t)H * 2);
    const __nv_bfloat16 *xp[P];
#pragma unroll
    for (int t = 0; t < P; ++t) xp[t] = a.x + (size_t)m.tok[qb + t] * H + lane * 8;
    float ag[P], au[P];
#pragma unroll
    for (int t = 0; t < P; ++t) {
        ag[t] = 0.f;
        au[t] = 0.f;
    }
#pragma unroll
    for (int c8 = 0; c8 < kGuChunks; ++c8) {
        const int c = c8 * 256 + lane * 8;
        if (c < H) {
            const uint4 wg = gs[c >> 3], wu = us[c >> 3];
            uint4 xv[P];
#pragma unroll
            for (int t = 0; t < P; ++t) xv[t] = ld_cached16(xp[t] + c8 * 256);
#pragma unroll
            for (int t = 0; t < P; ++t) {
                ag[t] = dot8(wg, xv[t], ag[t]);
                au[t] = dot8(wu, xv[t], au[t]);
            }
        }
    }
#pragma unroll
    for (int t = 0; t < P; ++t) {
        const float g = round_bf16(warp_sum(ag[t]));
        const float v = round_bf16(warp_sum(au[t]));
        if (lane == kPubLane) {  // one lane stores every pair's row j
            const float sg = silu_stored(g);
            st_relaxed_bf16(a.act + (size_t)m.pair[qb + t] * I + j, act_value(sg * v));
        }
    }
}

// Activation rows of up to CP pairs, kept in registers across the down units
// of one expert (CP 4 with 8 warps per block; 2 with 12, within their
// register budget).
template <int CP>
struct ActCache {
    uint4 v[CP][kDqChunks];
};

// One pass of a down unit over P pairs starting at list entry qb; `cache`
// holds the pairs' activation rows when the expert has at most kPairPass pairs.
template <int P, bool CACHED, int OFF = 0, int CP = kPairPass>
__device__ __forceinline__ void dn_pass(const GroupCompute &a, const Meta &m, int qb, const unsigned char *st,
                                        int h0, int nr, int lane, const ActCache<CP> &cache) {
    const int H = a.H, I = a.I;
    const uint4 *ws = reinterpret_cast<const uint4 *>(st);
    float acc[4][P];
#pragma unroll
    for (int t = 0; t < P; ++t)
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
            for (int t = 0; t < P; ++t) {
                const uint4 av = CACHED ? cache.v[OFF + t][c4] : ld_cg16(a.act + (size_t)m.pair[qb + t] * I + c);
#pragma unroll
                for (int r = 0; r < 4; ++r) acc[r][t] = dot8(wv[r], av, acc[r][t]);
            }
        }
    }
#pragma unroll
    for (int t = 0; t < P; ++t) {
        const int p = m.pair[qb + t];
        const float wp = m.wt[qb + t];
#pragma unroll
        for (int r = 0; r < 4; ++r) {
            const float sum = warp_sum(acc[r][t]);
            if (lane == r && r < nr) a.y[(size_t)p * H + h0 + r] = __float2bfloat16_rn(sum * wp);
        }
    }
}

// Until every activation row of expert u's pairs is written (no element still
// kActEmpty; each element is written once per launch by one 2-byte store), poll
// this lane's chunks of them (bounded).  With CACHED (at most kPairPass pairs)
// the rows land in `cache`.  Returns false when the kernel is aborting.
template <bool CACHED, int CP>
__device__ bool poll_act(const GroupCompute &a, const Meta &m, int q0, int np, int lane,
                         const ForwardParams &fp, ActCache<CP> &cache) {
    const int I = a.I;
    unsigned long long t0 = 0;
    volatile unsigned int *vabort = fp.bar + kBarAbort;
    for (int iter = 0;; ++iter) {
        bool full = true;
        if (CACHED) {
#pragma unroll
            for (int t = 0; t < CP; ++t)
                if (t < np)
#pragma unroll
                    for (int c4 = 0; c4 < kDqChunks; ++c4) {
                        const int c = c4 * 256 + lane * 8;
                        if (c < I) {
                            cache.v[t][c4] = ld_volatile16(a.act + (size_t)m.pair[q0 + t] * I + c);
                            full &= !has_empty(cache.v[t][c4]);
                        }
                    }
        } else {
            for (int t = 0; t < np; ++t)
#pragma unroll
                for (int c4 = 0; c4 < kDqChunks; ++c4) {
                    const int c = c4 * 256 + lane * 8;
                    if (c < I) full &= !has_empty(ld_volatile16(a.act + (size_t)m.pair[q0 + t] * I + c));
                }
        }
        if (__all_sync(0xffffffffu, full)) return true;
        int stop = 0;
        if (lane == 0) {
            if (iter == 0) t0 = globaltimer_ns();
            if (*vabort) {
                stop = 1;
            } else if ((long long)(globaltimer_ns() - t0) > fp.wait_ns) {
                set_status(fp.bar, WISP_ERR_TIMEOUT);
                atomicExch(fp.bar + kBarAbort, 1u);
                stop = 1;
            }
        }
        if (__shfl_sync(0xffffffffu, stop, 0)) return false;
        __nanosleep(128);
    }
}

// Run a warp's stream.  With `dataflow`, a down unit first polls until its
// expert's activation rows are complete (its W2 copy already in flight);
// without it the caller separates the phases with a grid barrier.  Down units
// store the weighted y; the row-quad arrivals are made later (arrive_stream).
// The gate-up items and the down items run in two tight loops (one compact
// body each); the copy pipeline runs on across the change.  Returns false
// when the kernel is aborting.
// Optional per-warp trace (debug; `wtr` null when off): [0] start, [1] first
// unit's data ready, [2] gate-up items done, [3] all items done, [4] ns in
// copy waits, [5] ns in activation polls, [6] items; %globaltimer.
template <int CP>
__device__ bool run_stream(const GroupCompute &a, const Meta &m, const Stream &S, int lane,
                           const ForwardParams &fp, WarpPipe &w, bool dataflow,
                           unsigned long long *wtr = nullptr) {
    const int H = a.H, I = a.I;
    const uint32_t rowb = (uint32_t)H * 2;
    unsigned long long t_copy = 0, t_act = 0;
    int units = 0;
    if (wtr && lane == 0) wtr[0] = globaltimer_ns();
    // copy the weights of the item under cursor c into stage s
    auto issue = [&](const Cursor &c, int s) -> bool {
        const int u = S.u0 + c.e;
        if (m.gen[u] != 0) {  // expert paged in during this call: its slot must have landed
            int ok = 1;
            if (lane == 0) ok = wait_slot(fp.slot_ready, m.slot[u], (uint32_t)m.gen[u], fp.bar, fp.wait_ns);
            if (!__shfl_sync(0xffffffffu, ok, 0)) return false;
        }
        if (lane == 0) {
            if (c.gu_left > 0) {
                const __nv_bfloat16 *g = a.w13 + (size_t)m.slot[u] * (size_t)(2 * I) * H + (size_t)c.r * H;
                pipe_issue(w, s, g, rowb, g + (size_t)I * H, rowb);
            } else {
                const int nr = min(4, H - 4 * c.r);
                pipe_issue(w, s, a.w2 + (size_t)m.slot[u] * (size_t)H * I + (size_t)(4 * c.r) * I,
                           (uint32_t)nr * I * 2, nullptr, 0);
            }
        }
        w.pending |= 1u << s;
        return true;
    };
    Cursor iss = cursor_begin(S), cmp = iss;
    bool ok = true;
    for (int s0 = 0; s0 < w.nst && ok && !iss.done; ++s0) {
        ok = issue(iss, s0);
        cursor_next(iss, S);
    }
    auto wait_stage = [&](int s) -> bool {
        const unsigned long long tw = wtr ? globaltimer_ns() : 0;
        if (!pipe_wait(w, s, fp)) return false;
        if (wtr) {
            t_copy += globaltimer_ns() - tw;
            if (units == 0 && lane == 0) wtr[1] = globaltimer_ns();
        }
        return true;
    };
    int s = 0;
    // ---- gate-up items
    while (ok && cmp.gu_left > 0) {
        const int u = S.u0 + cmp.e, j = cmp.r;
        const unsigned char *st = w.buf + s * kStageBytes;
        if (!wait_stage(s)) {
            ok = false;
            break;
        }
        int qb = m.off[u];
        const int q1 = m.off[u + 1];
        for (; qb + 4 <= q1; qb += 4) gu_pass<4>(a, m, qb, st, j, lane);
        if (qb + 2 <= q1) {
            gu_pass<2>(a, m, qb, st, j, lane);
            qb += 2;
        }
        if (qb < q1) gu_pass<1>(a, m, qb, st, j, lane);
        __syncwarp();
        ++units;
        if (!iss.done) {
            ok = issue(iss, s);
            cursor_next(iss, S);
        }
        cursor_next(cmp, S);
        s = (s + 1 == w.nst) ? 0 : s + 1;
    }
    if (wtr && lane == 0) wtr[2] = globaltimer_ns();
    // ---- down items
    ActCache<CP> cache;
    int cache_u = -1, ready_u = -1;
    while (ok && !cmp.done) {
        const int u = S.u0 + cmp.e, h0 = 4 * cmp.r, nr = min(4, H - h0);
        const int q0 = m.off[u], q1 = m.off[u + 1], np = q1 - q0;
        const unsigned char *st = w.buf + s * kStageBytes;
        const bool cached = np <= CP;
        if (dataflow && u != ready_u) {
            const unsigned long long ta = wtr ? globaltimer_ns() : 0;
            if (!(cached ? poll_act<true>(a, m, q0, np, lane, fp, cache)
                         : poll_act<false>(a, m, q0, np, lane, fp, cache))) {
                ok = false;
                break;
            }
            if (wtr) t_act += globaltimer_ns() - ta;
            ready_u = u;
            if (cached) cache_u = u;
        }
        if (cached && u != cache_u) {  // this expert's activation rows, reused by its next units
#pragma unroll
            for (int t = 0; t < CP; ++t)
                if (t < np)
#pragma unroll
                    for (int c4 = 0; c4 < kDqChunks; ++c4) {
                        const int c = c4 * 256 + lane * 8;
                        if (c < I) cache.v[t][c4] = ld_cg16(a.act + (size_t)m.pair[q0 + t] * I + c);
                    }
            cache_u = u;
        }
        if (!wait_stage(s)) {
            ok = false;
            break;
        }
        if (cached) {
            if constexpr (CP >= 4) {
                if (np == 4) {
                    dn_pass<4, true, 0, CP>(a, m, q0, st, h0, nr, lane, cache);
                } else {
                    if (np >= 2) dn_pass<2, true, 0, CP>(a, m, q0, st, h0, nr, lane, cache);
                    if (np == 3) dn_pass<1, true, 2, CP>(a, m, q0 + 2, st, h0, nr, lane, cache);
                    if (np == 1) dn_pass<1, true, 0, CP>(a, m, q0, st, h0, nr, lane, cache);
                }
            } else {
                if (np == 2) dn_pass<2, true, 0, CP>(a, m, q0, st, h0, nr, lane, cache);
                if (np == 1) dn_pass<1, true, 0, CP>(a, m, q0, st, h0, nr, lane, cache);
            }
        } else {
            int qb = q0;
            for (; qb + 4 <= q1; qb += 4) dn_pass<4, false, 0, CP>(a, m, qb, st, h0, nr, lane, cache);
            if (qb + 2 <= q1) {
                dn_pass<2, false, 0, CP>(a, m, qb, st, h0, nr, lane, cache);
                qb += 2;
            }
            if (qb < q1) dn_pass<1, false, 0, CP>(a, m, qb, st, h0, nr, lane, cache);
        }
        __syncwarp();
        ++units;
        if (!iss.done) {
            ok = issue(iss, s);
            cursor_next(iss, S);
        }
        cursor_next(cmp, S);
        s = (s + 1 == w.nst) ? 0 : s + 1;
    }
    if (!ok) {
        pipe_drain(w, fp);
        return false;
    }
    if (wtr && lane == 0) {
        wtr[3] = globaltimer_ns();
        wtr[4] = t_copy;
        wtr[5] = t_act;
        wtr[6] = (unsigned long long)units;
    }
    return true;
}

__device__ __forceinline__ int atom_add_acq_rel_gpu(int32_t *p, int v) {
    int old;
    asm volatile("atom.acq_rel.gpu.global.add.s32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
    return old;
}

// Row-quad arrivals of a warp's down units (after their y stores): one lane
// per unit counts itself in with an acquire-release atomic at GPU scope (after
// a warp barrier, so the other lanes' y stores are released too); the units
// that complete their quad (the nu-th arrival) then sum the group's tokens
// over k in routing order for those rows, all of them in one pass over the
// warp's lanes (one output per lane, its K loads in flight together).
__device__ void arrive_stream(const GroupCompute &a, const Stream &S, int nu, int lane) {
    if (S.n_dn == 0 || S.j0 >= S.nch) return;
    const int per = (a.t1 - a.t0) * 4;  // outputs of one row quad
    // this warp's down units, 32 at a time (lane l takes the l-th)
    int j = S.j0, d = j * kDownChunk;
    while (j < S.nch) {
        int mine = -1;
        for (int l = 0; l < 32 && j < S.nch; ++l) {
            if (l == lane) mine = d;
            if (++d >= min((j + 1) * kDownChunk, S.n_dn)) {
                j += S.nw;
                d = j * kDownChunk;
            }
        }
        __syncwarp();
        int last = 0, q = 0;
        if (mine >= 0) {
            q = mine % S.nq;
            last = atom_add_acq_rel_gpu(&a.counters[q], 1) == nu - 1;
        }
        const unsigned todo = __ballot_sync(0xffffffffu, last);
        __syncwarp();
        const int n = __popc(todo) * per;
        for (int i0 = 0; i0 < n; i0 += 32) {
            const int idx = i0 + lane;
            const int which = idx < n ? idx / per : 0;
            unsigned m = todo;
            for (int i = 0; i < which; ++i) m &= m - 1;
            const int qv = __shfl_sync(0xffffffffu, q, m ? __ffs(m) - 1 : 0);
            if (idx < n) {
                const int rem = idx - which * per;
                const int hh = qv * 4 + (rem & 3);
                if (hh < a.H) combine_one(a, a.t0 + (rem >> 2), hh);
            }
        }
        if (last) a.counters[q] = 0;
    }
}

// The last of the nu units of row quad q to finish sums the group's tokens
// (generic variant).
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
// `pos` is scratch for 2 E ints (the second half holds a copy of the expert
// map, loaded together with the routing ids: one global round trip).
__device__ bool build_spec_meta(const ForwardParams &fp, Meta &m, int *pos) {
    __shared__ uint32_t s_mask[32];
    __shared__ int s_flag;
    __shared__ int s_fill[kMetaU];
    const PagerParams &pg = fp.pg;
    const int P = pg.T * pg.K, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    if (P > kSpecMaxPairs || pg.E > 1024) return false;
    int *s_emap = pos + pg.E;
    // this thread's routed id (P <= kSpecMaxPairs <= blockDim.x) in flight
    // together with the map: one global round trip
    const long long my_e = tid < P ? load_id64(pg.ids, pg.ids64, tid) : 0;
    const float my_w = tid < P ? fp.gc.topk_w[tid] : 0.f;
    if (tid < 32) s_mask[tid] = 0;
    if (tid == 0) s_flag = 0;
    for (int e = tid; e < pg.E; e += blockDim.x) s_emap[e] = pg.emap[e];
    __syncthreads();
    for (int p = tid; p < P; p += blockDim.x) {
        const long long e = my_e;
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
            if (s_emap[lane * 32 + b] >= 0) keep |= 1u << b;
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
            m.slot[idx] = s_emap[e];
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
            m.total = total;
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
        m.wt[at] = my_w;
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
        m.wt[i] = fp.gc.topk_w[p];
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
// I <= 1024): TMA-fed warp streams, a speculative start, and for a call that
// forms one token group no grid barrier at all (down units poll the
// activation rows they need).  Otherwise the generic bodies with grid
// barriers between phases.  The host picks the variant from the shapes alone.
template <int MAXP, bool FAST, int NW>
__global__ void __launch_bounds__(NW * 32, kBlocksPerSm) forward_kernel(const __grid_constant__ ForwardParams a) {
    extern __shared__ __align__(16) unsigned char smem[];
    __shared__ Meta meta;
    constexpr int MAXQ = MAXP < 4 ? MAXP : 4;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, tid = threadIdx.x;
    const int nwarps = gridDim.x * NW;
    const int gw = blockIdx.x * NW + warp;
    const PagerParams &pg = a.pg;
    const int H = a.gc.H, I = a.gc.I, nq = (H + 3) / 4;
    constexpr int CP = NW > kWarpsDeep ? 2 : kPairPass;  // activation-cache pairs (register budget)
    unsigned long long *tr = a.trace;
#define WISP_TRACE(slot)                                                                 \
    do {                                                                                 \
        if (tr && tid == 0) tr[8 + blockIdx.x * 4 + (slot)] = globaltimer_ns();          \
    } while (0)
#define WISP_TRACE0(slot)                                                                \
    do {                                                                                 \
        if (tr && tid == 0 && blockIdx.x == 0) tr[(slot)] = globaltimer_ns();            \
    } while (0)
    pdl_wait();
    pdl_launch_dependents();
    WISP_TRACE(0);
    WISP_TRACE0(0);

    // per-warp copy pipelines (FAST variant); buffers overlay the pager's shared
    // memory, which block 0 is done with before its first copy
    __shared__ __align__(8) uint64_t s_bars[NW][kMaxStages];
    WarpPipe pipe{};
    if (FAST) {
        pipe.nst = a.stages;
        pipe.buf = smem + (size_t)warp * a.stages * kStageBytes;
        pipe.bar = s_bars[warp];
        pipe.pol = l2_evict_first_policy();
        if (lane == 0) {
            for (int st = 0; st < a.stages; ++st) mbar_init(pipe.bar + st, 1);
            fence_proxy_async();
        }
        __syncwarp();
    }

    // ---- phase 0 ------------------------------------------------------------------
    // block 0: pager, publish its outputs, wait until no block still reads the
    // pre-call expert map, write the new state back.  Other blocks: read the
    // pre-call map (speculation lists), say so, and run the gate-up and down
    // units of the experts that were resident before the call (their row-quad
    // arrivals wait until the call's expert count is known).
    Stream spec{};
    if (blockIdx.x == 0) {
        if (tid == 0) a.flow[kFlowSpecRead + (a.epoch ^ 1)] = 0;  // the next launch's count starts at zero
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
        bool spec_here = false;
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
            spec = make_stream(0, meta.nu, true, true, gw - NW, nwarps - NW, I, nq);
            // (an abort shows in the next wait)
            run_stream<CP>(gc, meta, spec, lane, a, pipe, true, tr ? tr + kTraceWarps + gw * 16 : nullptr);
        }
        // every expert of the call was resident before it: the pager will find
        // one group of hits only, so nothing is left but the speculative
        // stream's row-quad arrivals; the warps of this block make them and
        // leave without waiting for the pager or for each other (the condition
        // is the same for every warp of the block)
        if (spec_here && meta.total == meta.nu) {
            GroupCompute gc = a.gc;
            gc.t0 = 0;
            gc.t1 = pg.T;
            arrive_stream(gc, spec, meta.nu, lane);
            if (tr && lane == 0) tr[kTraceWarps + gw * 16 + 7] = globaltimer_ns();
            WISP_TRACE(3);
            goto done;
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
            const Stream rest = make_stream(u_lo, nu, true, true, gw, nwarps, I, nq);
            if (!run_stream<CP>(gc, meta, rest, lane, a, pipe, true, tr ? tr + kTraceWarps + gw * 16 + 8 : nullptr))
                goto done;
            WISP_TRACE(2);
            arrive_stream(gc, spec, nu, lane);
            arrive_stream(gc, rest, nu, lane);
            if (tr && lane == 0) tr[kTraceWarps + gw * 16 + 7] = globaltimer_ns();
            __syncthreads();
            WISP_TRACE(3);
        } else {
            // ---- several groups (or the generic variant): grid barriers between phases ---------
            if (!grid_barrier(a.bar, a.wait_ns)) goto done;
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
                    run_stream<CP>(gc, meta, make_stream(0, nu, true, false, gw, nwarps, I, nq), lane, a, pipe,
                               false);
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
                    const Stream dn = make_stream(0, nu, false, true, gw, nwarps, I, nq);
                    if (run_stream<CP>(gc, meta, dn, lane, a, pipe, false)) arrive_stream(gc, dn, nu, lane);
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
    }
done:
    // the next launch's activation buffer: every element "not written yet"
    // (after this launch's work, so these stores do not hold up its fences;
    // every block gets here, aborts included)
    for (long i = (long)blockIdx.x * (NW * 32) + tid; i < a.act_reset_words; i += (long)gridDim.x * (NW * 32))
        a.act_reset[i] = 0xFFFFFFFFu;
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

template <int MAXP, bool FAST, int NW>
int launch_t(const ForwardParams &p, size_t smem, cudaStream_t stream) {
    static int nblk_per_sm[64];
    static size_t smem_set[64];
    int dev = 0;
    WISP_CUDA_TRY(cudaGetDevice(&dev));
    if (dev < 0 || dev >= 64) return WISP_ERR_INVALID;
    if (smem_set[dev] < smem || !nblk_per_sm[dev]) {
        WISP_CUDA_TRY(cudaFuncSetAttribute(forward_kernel<MAXP, FAST, NW>,
                                           cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
        int nb = 0;
        WISP_CUDA_TRY(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&nb, forward_kernel<MAXP, FAST, NW>, NW * 32, smem));
        if (nb < 1) return set_error("forward kernel does not fit on an SM"), WISP_ERR_UNSUPPORTED;
        nblk_per_sm[dev] = nb > kBlocksPerSm ? kBlocksPerSm : nb;
        smem_set[dev] = smem;
    }
    int sms = 0;
    WISP_CUDA_TRY(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
    dim3 grid(sms * nblk_per_sm[dev]), block(NW * 32);
    return launch_persistent(forward_kernel<MAXP, FAST, NW>, grid, block, smem, stream, p);
}

}  // namespace

int launch_forward(const ForwardParams &p, int max_tokens_per_group, cudaStream_t stream) {
    size_t smem = pager_smem_bytes(p.pg.E, p.pg.cap, p.pg.T, p.pg.K);
    smem = smem > sizeof(int) * 2048 ? smem : sizeof(int) * 2048;  // speculation's expert index + map
    const bool fast = (long)p.pg.T * p.pg.K <= kMetaP && p.gc.H <= kGuChunks * 256 &&
                      p.gc.I <= kDqChunks * 256 && 2L * 2 * p.gc.H <= kStageBytes &&
                      4L * 2 * p.gc.I <= kStageBytes;
    if (fast) {
        ForwardParams q = p;
        if ((long)p.pg.T * p.pg.K <= 8) {  // one token: 8 warps x 3 stages
            q.stages = 3;
            const size_t st = (size_t)kWarpsDeep * 3 * kStageBytes;
            return launch_t<1, true, kWarpsDeep>(q, smem > st ? smem : st, stream);
        }
        q.stages = 2;  // 12 warps x 2 stages
        const size_t st = (size_t)kWarpsWide * 2 * kStageBytes;
        return launch_t<1, true, kWarpsWide>(q, smem > st ? smem : st, stream);
    }
    if (max_tokens_per_group <= 1) return launch_t<1, false, kWarpsDeep>(p, smem, stream);
    if (max_tokens_per_group <= 4) return launch_t<4, false, kWarpsDeep>(p, smem, stream);
    return launch_t<8, false, kWarpsDeep>(p, smem, stream);
}

}  // namespace wisp
