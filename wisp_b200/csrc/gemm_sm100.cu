// Prefill expert compute for one token group on tcgen05 tensor cores; see
// gemm_sm100.cuh for the data flow and the kernel structure.
#include "gemm_sm100.cuh"
#include "pager.cuh"
#include "prefill.cuh"

#include <algorithm>
#include <mutex>

namespace wisp {
namespace gemm {
namespace {

__device__ __forceinline__ unsigned char *align1024(unsigned char *p) {
    const uint32_t a = s_addr(p);
    return p + ((1024u - (a & 1023u)) & 1023u);
}

// X_perm[q] = x[token of pair q]: one warp per row, 16-byte copies.  When
// the pager ran without a host check and rejected the call, the lists are
// stale: nothing is read and block 0 records the pager's status in the
// sticky word.
__global__ void gather_kernel(const uint4 *x, const int32_t *u_pairs, int P, int K, int H8, uint4 *xp,
                              const int32_t *pager_status, int *status) {
    pdl_wait();
    pdl_launch_dependents();
    if (pager_status) {
        const int st = *reinterpret_cast<const volatile int32_t *>(pager_status);
        if (st != WISP_OK) {
            if (blockIdx.x == 0 && threadIdx.x == 0 && status) *reinterpret_cast<volatile int *>(status) = st;
            return;
        }
    }
    const int q = blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5);
    if (q >= P) return;
    const uint4 *src = x + (size_t)(u_pairs[q] / K) * H8;
    uint4 *dst = xp + (size_t)q * H8;
    for (int c = threadIdx.x & 31; c < H8; c += 32) dst[c] = src[c];
}

// ---- routing and gather of a resident call (one cooperative launch) ---------------
// Counting sort of the call's P pairs by expert, fused with the gather of
// their token rows.  Block b takes the contiguous pairs [b R, (b + 1) R):
//   1. counts them per expert in shared memory and adds the counts to the
//      launch's global per-expert counters (ids outside [0, E) raise a flag);
//   2. grid barrier;
//   3. every block scans the global counts over the experts (first list
//      position of each expert; block 0 writes the lists' header: offsets,
//      slots, the expert count, the header words and the forward's count);
//      each block reserves its run inside every expert's range with one
//      global atomic per expert it holds, then places its pairs (shared
//      atomics) and copies their token rows x[t] to X_perm[position].
// The experts appear in ascending order; the order of one expert's pairs is
// the order the atomics ran, which changes no output bit (each pair's row is
// computed on its own, and the combine indexes rows by pair).  The counters
// come in two halves by launch parity: a launch uses one (zero on entry) and
// zeroes the other for the next launch.
constexpr int kRouteThreads = 1024;
constexpr int kRouteMaxExperts = 1024;
constexpr int kRouteExpertsPerThread = kRouteMaxExperts / kRouteThreads;
struct RouteArgs {
    const void *ids;
    int ids64, P, E, K, H8, count_forward;
    const int32_t *emap;
    const uint4 *x;
    uint4 *x_perm;
    int64_t *hdr;
    int32_t *dev_hdr;
    int *status;                      // sticky status word
    int32_t *u_off, *u_pairs, *u_slot, *nu;
    int32_t *cnt, *cnt_next;          // [2 E + 1]: counts, fills, bad-id flag
    uint32_t *bar;                    // [2]: arrivals, generation (self-resetting)
    long long wait_ns;
};

// Routed id of pair p: the expert, or -1 when outside [0, E).
__device__ __forceinline__ int route_id(const RouteArgs &r, int p) {
    const long long e = load_id64(r.ids, r.ids64, p);
    return (e < 0 || e >= r.E) ? -1 : (int)e;
}

__device__ __forceinline__ int block_excl_scan(int v, int *s_warp, int &total) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    int inc = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int t = __shfl_up_sync(0xffffffffu, inc, o);
        if (lane >= o) inc += t;
    }
    if (lane == 31) s_warp[warp] = inc;
    __syncthreads();
    if (warp == 0) {
        int w = lane < (int)(blockDim.x >> 5) ? s_warp[lane] : 0;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int t = __shfl_up_sync(0xffffffffu, w, o);
            if (lane >= o) w += t;
        }
        s_warp[lane] = w;  // inclusive over warps
    }
    __syncthreads();
    total = s_warp[(blockDim.x >> 5) - 1];
    const int before = warp > 0 ? s_warp[warp - 1] : 0;
    __syncthreads();  // s_warp is reused by the next scan
    return before + inc - v;
}

// Every block; false when the wait ran out (then the status word says so).
__device__ bool route_grid_barrier(const RouteArgs &r) {
    __shared__ int s_ok;
    __syncthreads();
    if (threadIdx.x == 0) {
        volatile uint32_t *vgen = r.bar + 1;
        const uint32_t gen = *vgen;
        __threadfence();
        int ok = 1;
        if (atomicAdd(r.bar, 1u) == gridDim.x - 1) {
            atomicExch(r.bar, 0u);
            __threadfence();
            atomicAdd(r.bar + 1, 1u);
        } else {
            const unsigned long long t0 = globaltimer_ns();
            while (*vgen == gen) {
                if ((long long)(globaltimer_ns() - t0) > r.wait_ns) {
                    ok = 0;
                    break;
                }
                __nanosleep(64);
            }
        }
        __threadfence();
        s_ok = ok;
    }
    __syncthreads();
    return s_ok != 0;
}

__global__ void __launch_bounds__(kRouteThreads, 1) route_gather_kernel(const RouteArgs r) {
    extern __shared__ int2 route_list[];  // this block's (pair, expert), then (pair, position)
    __shared__ int hist[kRouteMaxExperts];  // this block's pairs per expert, then its next place
    __shared__ int eoff[kRouteMaxExperts];
    __shared__ int s_warp[32];
    __shared__ int s_bad;
    const int E = r.E, P = r.P, tid = threadIdx.x;
    pdl_wait();
    pdl_launch_dependents();
    const int R = (P + gridDim.x - 1) / gridDim.x;
    const int p_lo = min(P, (int)blockIdx.x * R), p_hi = min(P, p_lo + R), n = p_hi - p_lo;
    for (int e = tid; e < E; e += kRouteThreads) hist[e] = 0;
    for (int i = blockIdx.x * kRouteThreads + tid; i < 2 * E + 1; i += gridDim.x * kRouteThreads)
        r.cnt_next[i] = 0;
    if (tid == 0) s_bad = 0;
    __syncthreads();
    for (int i = tid; i < n; i += kRouteThreads) {
        const int e = route_id(r, p_lo + i);
        route_list[i] = make_int2(p_lo + i, e);
        if (e < 0)
            s_bad = 1;
        else
            atomicAdd(&hist[e], 1);
    }
    __syncthreads();
    if (s_bad && tid == 0) atomicOr(r.cnt + 2 * E, 1);
    for (int e = tid; e < E; e += kRouteThreads)
        if (hist[e]) atomicAdd(r.cnt + e, hist[e]);
    const bool synced = route_grid_barrier(r);
    if (!synced || *reinterpret_cast<volatile int32_t *>(r.cnt + 2 * E)) {
        if ((blockIdx.x == 0 || !synced) && tid == 0) {  // a block whose wait ran out reports it itself
            const int code = synced ? WISP_ERR_BAD_EXPERT : WISP_ERR_TIMEOUT;
            *reinterpret_cast<volatile int32_t *>(r.dev_hdr + kHdrStatus) = code;
            if (r.status) *reinterpret_cast<volatile int *>(r.status) = code;
        }
        return;  // the call's other kernels see the status and do nothing
    }
    // experts [4 tid, 4 tid + 4): counts, then offsets and unique indices by block scans
    int c[kRouteExpertsPerThread], f = 0, sum = 0;
#pragma unroll
    for (int j = 0; j < kRouteExpertsPerThread; ++j) {
        const int e = tid * kRouteExpertsPerThread + j;
        c[j] = e < E ? __ldcg(r.cnt + e) : 0;
        sum += c[j];
        f += c[j] > 0;
    }
    int nu = 0, ptot = 0;
    int u = block_excl_scan(f, s_warp, nu);
    int off = block_excl_scan(sum, s_warp, ptot);
#pragma unroll
    for (int j = 0; j < kRouteExpertsPerThread; ++j) {
        const int e = tid * kRouteExpertsPerThread + j;
        if (e < E) {
            eoff[e] = off;
            if (blockIdx.x == 0 && c[j] > 0) {
                r.u_off[u] = off;
                r.u_slot[u] = r.emap[e];
            }
        }
        off += c[j];
        u += c[j] > 0;
    }
    if (blockIdx.x == 0 && tid == 0) {
        r.u_off[nu] = P;
        *r.nu = nu;
        r.dev_hdr[kHdrGroups] = 1;
        r.dev_hdr[kHdrMisses] = 0;
        r.dev_hdr[kHdrUnique] = nu;
        if (r.count_forward) r.hdr[1] += 1;  // the forward (resident layers count only that)
        r.hdr[5] += 1;                       // telemetry: groups, unique experts
        r.hdr[6] += nu;
        r.dev_hdr[kHdrStatus] = WISP_OK;
    }
    __syncthreads();
    // this block's run inside each expert's range
    for (int e = tid; e < E; e += kRouteThreads)
        if (hist[e]) hist[e] = eoff[e] + atomicAdd(r.cnt + E + e, hist[e]);
    __syncthreads();
    for (int i = tid; i < n; i += kRouteThreads) {
        const int2 pe = route_list[i];
        const int pos = atomicAdd(&hist[pe.y], 1);
        r.u_pairs[pos] = pe.x;
        route_list[i] = make_int2(pe.x, pos);
    }
    __syncthreads();
    // token rows: warp w copies rows w, w + 32, ..., two rows at a time with
    // up to 8 16-byte words of each in flight per lane (32-bit index arithmetic)
    const int H8 = r.H8, K = r.K, lane = tid & 31, warp = tid >> 5;
    constexpr int kWarpsR = kRouteThreads / 32;
    for (int r0 = warp; r0 < n; r0 += 2 * kWarpsR) {
        const int r1 = r0 + kWarpsR;
        const int2 a = route_list[r0];
        const int2 b = r1 < n ? route_list[r1] : make_int2(0, -1);
        const uint4 *sa = r.x + (size_t)(a.x / K) * H8, *sb = r.x + (size_t)(b.x / K) * H8;
        uint4 *da = r.x_perm + (size_t)a.y * H8, *db = r.x_perm + (size_t)(b.y < 0 ? 0 : b.y) * H8;
        for (int w0 = lane; w0 < H8; w0 += 32 * 4) {
            uint4 va[4], vb[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const int w = w0 + 32 * j;
                if (w < H8) {
                    va[j] = __ldg(sa + w);
                    if (b.y >= 0) vb[j] = __ldg(sb + w);
                }
            }
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const int w = w0 + 32 * j;
                if (w < H8) {
                    da[w] = va[j];
                    if (b.y >= 0) db[w] = vb[j];
                }
            }
        }
    }
}

// The group's experts and their 128-pair tiles, in shared memory.
constexpr int kMaxTileExperts = 1024;
struct TileTable {
    int nu, mtiles;
    int off[kMaxTileExperts + 1];  // pair-list offsets
    int mt[kMaxTileExperts + 1];   // first tile of each expert (prefix of tile counts)
};

// Tile m -> expert u, first list position q0, rows (binary search: the last
// expert whose first tile is <= m; every expert of a group has pairs).
__device__ __forceinline__ void tile_of(const TileTable &tt, int m, int &u, int &q0, int &rows) {
    int lo = 0, hi = tt.nu - 1;
    while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (tt.mt[mid] <= m)
            lo = mid;
        else
            hi = mid - 1;
    }
    u = lo;
    q0 = tt.off[u] + (m - tt.mt[u]) * kBM;
    rows = min(kBM, tt.off[u + 1] - q0);
}

// Setup of a persistent GEMM CTA: tile table, barriers, TMEM (both
// accumulators).  Returns the number of tiles (n_cols tiles per m tile); a CTA
// with none returns 0 before allocating anything.
__device__ __forceinline__ int gemm_setup(const GroupGemm &g, int n_cols, TileTable &tt, Ring &R) {
    const int nu = min(group_experts(g.nu_dev, g.pager_status), kMaxTileExperts);
    for (int i = threadIdx.x; i <= nu; i += blockDim.x) tt.off[i] = g.u_off[i];
    __syncthreads();
    if (threadIdx.x == 0) {
        tt.nu = nu;
        int acc = 0;
        for (int e = 0; e < nu; ++e) {
            tt.mt[e] = acc;
            acc += (tt.off[e + 1] - tt.off[e] + kBM - 1) / kBM;
        }
        tt.mt[nu] = acc;
        tt.mtiles = acc;
        R.abort = 0;
        R.issued = R.consumed = 0;
        for (int s = 0; s < kStages; ++s) {
            mbar_init(&R.full[s], 1);
            mbar_init(&R.empty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&R.acc_full[b], 1);
            mbar_init(&R.acc_empty[b], kEpiThreads);
        }
        mbar_init(&R.mma_done, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    }
    __syncthreads();
    const int ntiles = tt.mtiles * n_cols;
    if ((int)blockIdx.x >= ntiles) return 0;
    if ((threadIdx.x >> 5) == 0) tmem_alloc(&R.tmem_base, kTmemCols);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    return ntiles;
}

__device__ __forceinline__ void gemm_teardown(Ring &R, const GroupGemm &g) {
    tc_fence_before();
    __syncthreads();
    if (R.abort) drain_ring(R, g);
    __syncthreads();
    tc_fence_after();
    if ((threadIdx.x >> 5) == 0) tmem_dealloc(R.tmem_base, kTmemCols);
}

// Epilogue side of tile i (warps 2..5): wait for its accumulator; false after
// an abort.  Uniform over the warp, which leaves converged for the
// .sync.aligned TMEM loads.
__device__ __forceinline__ bool wait_acc(Ring &R, int i, const GroupGemm &g) {
    volatile int *abort = &R.abort;
    const bool ok = mbar_wait(&R.acc_full[i & 1], (i / 2) & 1, g.wait_ns, abort) && !*abort;
    const bool all = __all_sync(0xffffffffu, ok);
    tc_fence_after();
    return all;
}
__device__ __forceinline__ void release_acc(Ring &R, int i) {
    tc_fence_before();
    mbar_arrive(&R.acc_empty[i & 1]);
}

// Gate-up + SiLU-mul, persistent: tiles (m, n) with n over I / 128 fastest.
__global__ void __launch_bounds__(kThreads, 1)
    gateup_gemm_kernel(const __grid_constant__ CUtensorMap map_x, const __grid_constant__ CUtensorMap map_w13,
                       GroupGemm g) {
    extern __shared__ unsigned char smem_raw[];
    __shared__ Ring R;
    __shared__ TileTable tt;
    unsigned char *stages = align1024(smem_raw);
    pdl_wait();
    pdl_launch_dependents();
    const int I = g.I, n_cols = I / kHalfN;
    const int ntiles = gemm_setup(g, n_cols, tt, R);
    if (ntiles == 0) return;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int kb_count = g.H / kBK;
    if (warp == 0) {
        if (lane == 0)
            produce(&map_x, &map_w13, ntiles, kb_count, stages, R, g, [&](int t) {
                int u, q0, rows;
                tile_of(tt, t / n_cols, u, q0, rows);
                const int slot_row = g.u_slot[u] * 2 * I, j0 = (t % n_cols) * kHalfN;
                return TileOperands{q0, slot_row + j0, slot_row + I + j0};
            });
    } else if (warp == 1) {
        if (lane == 0) issue_mmas(ntiles, kb_count, stages, R, g);
    } else {
        const int quarter = warp & 3, row = quarter * 32 + lane;
        int i = 0;
        for (int t = blockIdx.x; t < ntiles; t += gridDim.x, ++i) {
            if (!wait_acc(R, i, g)) break;
            int u, q0, rows;
            tile_of(tt, t / n_cols, u, q0, rows);
            const int j0 = (t % n_cols) * kHalfN;
            const uint32_t tbase = R.tmem_base + (i & 1) * kAccCols + ((uint32_t)(quarter * 32) << 16);
            __nv_bfloat16 *dst = g.act_perm + (size_t)(q0 + row) * I + j0;
            for (int c0 = 0; c0 < kHalfN; c0 += 32) {
                uint32_t gr[32], ur[32];
                tmem_ld32(tbase + c0, gr);
                tmem_ld32(tbase + kHalfN + c0, ur);
                if (row < rows) {
                    uint32_t packed[16];
#pragma unroll
                    for (int k = 0; k < 32; k += 2) {
                        float o[2];
#pragma unroll
                        for (int h = 0; h < 2; ++h) {
                            const float gv = round_bf16(__uint_as_float(gr[k + h]));
                            const float uv = round_bf16(__uint_as_float(ur[k + h]));
                            o[h] = silu_stored(gv) * uv;
                        }
                        packed[k / 2] = (uint32_t)__bfloat16_as_ushort(act_value(o[0])) |
                                        ((uint32_t)__bfloat16_as_ushort(act_value(o[1])) << 16);
                    }
                    uint4 *d4 = reinterpret_cast<uint4 *>(dst + c0);
#pragma unroll
                    for (int v = 0; v < 4; ++v)
                        d4[v] = make_uint4(packed[4 * v], packed[4 * v + 1], packed[4 * v + 2], packed[4 * v + 3]);
                }
            }
            release_acc(R, i);
        }
    }
    gemm_teardown(R, g);
}

// Down x routing weight, persistent: tiles (m, n) with n over H / 256 fastest.
__global__ void __launch_bounds__(kThreads, 1)
    down_gemm_kernel(const __grid_constant__ CUtensorMap map_act, const __grid_constant__ CUtensorMap map_w2,
                     GroupGemm g) {
    extern __shared__ unsigned char smem_raw[];
    __shared__ Ring R;
    __shared__ TileTable tt;
    unsigned char *stages = align1024(smem_raw);
    pdl_wait();
    pdl_launch_dependents();
    const int H = g.H, n_cols = H / kBN;
    const int ntiles = gemm_setup(g, n_cols, tt, R);
    if (ntiles == 0) return;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int kb_count = g.I / kBK;
    if (warp == 0) {
        if (lane == 0)
            produce(&map_act, &map_w2, ntiles, kb_count, stages, R, g, [&](int t) {
                int u, q0, rows;
                tile_of(tt, t / n_cols, u, q0, rows);
                const int slot_row = g.u_slot[u] * H, n0 = (t % n_cols) * kBN;
                return TileOperands{q0, slot_row + n0, slot_row + n0 + kHalfN};
            });
    } else if (warp == 1) {
        if (lane == 0) issue_mmas(ntiles, kb_count, stages, R, g);
    } else {
        const int quarter = warp & 3, row = quarter * 32 + lane;
        int i = 0;
        for (int t = blockIdx.x; t < ntiles; t += gridDim.x, ++i) {
            if (!wait_acc(R, i, g)) break;
            int u, q0, rows;
            tile_of(tt, t / n_cols, u, q0, rows);
            const int n0 = (t % n_cols) * kBN;
            const uint32_t tbase = R.tmem_base + (i & 1) * kAccCols + ((uint32_t)(quarter * 32) << 16);
            const int p = row < rows ? g.u_pairs[q0 + row] : 0;
            const float wp = row < rows ? g.topk_w[p] : 0.f;
            __nv_bfloat16 *dst = g.y + (size_t)p * H + n0;
            for (int c0 = 0; c0 < kBN; c0 += 32) {
                uint32_t r[32];
                tmem_ld32(tbase + c0, r);
                if (row < rows) {
                    uint32_t packed[16];
#pragma unroll
                    for (int k = 0; k < 32; k += 2)
                        packed[k / 2] =
                            (uint32_t)__bfloat16_as_ushort(__float2bfloat16_rn(__uint_as_float(r[k]) * wp)) |
                            ((uint32_t)__bfloat16_as_ushort(__float2bfloat16_rn(__uint_as_float(r[k + 1]) * wp))
                             << 16);
                    uint4 *d4 = reinterpret_cast<uint4 *>(dst + c0);
#pragma unroll
                    for (int v = 0; v < 4; ++v)
                        d4[v] = make_uint4(packed[4 * v], packed[4 * v + 1], packed[4 * v + 2], packed[4 * v + 3]);
                }
            }
            release_acc(R, i);
        }
    }
    gemm_teardown(R, g);
}

// out[t] = sum over k in routing order of y[t * K + k], t in [t0, t1).
__global__ void combine_kernel(const uint4 *y, int t0, int t1, int K, int H8, uint4 *out,
                               const int32_t *pager_status) {
    pdl_wait();
    pdl_launch_dependents();
    if (pager_status && *reinterpret_cast<const volatile int32_t *>(pager_status) != WISP_OK) return;
    const long i = (long)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (long)(t1 - t0) * H8) return;
    const int t = t0 + (int)(i / H8), c = (int)(i % H8);
    float acc[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[j] = 0.f;
    for (int k = 0; k < K; ++k) {
        const uint4 v = y[((size_t)t * K + k) * H8 + c];
        const uint32_t wv[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            acc[2 * j] = combine_add(acc[2 * j], bf16lo(wv[j]), K);
            acc[2 * j + 1] = combine_add(acc[2 * j + 1], bf16hi(wv[j]), K);
        }
    }
    uint32_t o[4];
#pragma unroll
    for (int j = 0; j < 4; ++j)
        o[j] = (uint32_t)__bfloat16_as_ushort(__float2bfloat16_rn(acc[2 * j])) |
               ((uint32_t)__bfloat16_as_ushort(__float2bfloat16_rn(acc[2 * j + 1])) << 16);
    out[(size_t)t * H8 + c] = make_uint4(o[0], o[1], o[2], o[3]);
}

// ---- host ----------------------------------------------------------------------
typedef CUresult (*EncodeTiledFn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                  const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
EncodeTiledFn g_encode = nullptr;
std::once_flag g_encode_once;

void init_encode() {
    void *fn = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess && fn)
        g_encode = reinterpret_cast<EncodeTiledFn>(fn);
    else
        cudaGetLastError();
}

}  // namespace

int make_map(CUtensorMap *map, const void *base, uint64_t rows, uint64_t cols, uint32_t box_rows) {
    std::call_once(g_encode_once, init_encode);
    if (!g_encode) return set_error("wisp: cuTensorMapEncodeTiled is not available"), WISP_ERR_UNSUPPORTED;
    const cuuint64_t dims[2] = {cols, rows};
    const cuuint64_t strides[1] = {cols * 2};
    const cuuint32_t box[2] = {(cuuint32_t)kBK, (cuuint32_t)box_rows};
    const cuuint32_t estr[2] = {1, 1};
    const CUresult r = g_encode(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void *>(base), dims, strides,
                                box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                                CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return set_error("wisp: cuTensorMapEncodeTiled failed"), WISP_ERR_CUDA;
    return WISP_OK;
}

int launch_gather(const PrefillGroup &p, cudaStream_t stream) {
    const int warps = 8;
    const int blocks = (p.npairs + warps - 1) / warps;
    if (blocks <= 0) return WISP_OK;
    return launch_chained(gather_kernel, dim3(blocks), dim3(warps * 32), 0, stream,
                          reinterpret_cast<const uint4 *>(p.x), p.u_pairs, p.npairs, p.K, p.H / 8,
                          reinterpret_cast<uint4 *>(p.x_perm), p.pager_status, p.status);
}

int launch_combine(const PrefillGroup &p, cudaStream_t stream) {
    const long n = (long)(p.t1 - p.t0) * (p.H / 8);
    if (n <= 0) return WISP_OK;
    return launch_chained(combine_kernel, dim3((unsigned)((n + 255) / 256)), dim3(256), 0, stream,
                          reinterpret_cast<const uint4 *>(p.y), p.t0, p.t1, p.K, p.H / 8,
                          reinterpret_cast<uint4 *>(p.out), p.pager_status);
}

}  // namespace gemm

bool prefill_shapes_supported(int H, int I) {
    return H > 0 && I > 0 && H % gemm::kBN == 0 && I % gemm::kHalfN == 0;
}

namespace {
int launch_prefill_kernels(const PrefillGroup &p, bool gather, cudaStream_t stream) {
    using namespace gemm;
    if (!prefill_shapes_supported(p.H, p.I))
        return set_error("wisp: prefill GEMM needs hidden % 256 == 0 and inter % 128 == 0"), WISP_ERR_UNSUPPORTED;
    if (p.npairs <= 0 || p.nu <= 0) return WISP_OK;
    static bool attr_set[64] = {};
    int dev = 0;
    WISP_CUDA_TRY(cudaGetDevice(&dev));
    if (dev < 0 || dev >= 64) return WISP_ERR_INVALID;
    if (!attr_set[dev]) {
        WISP_CUDA_TRY(cudaFuncSetAttribute(gateup_gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes));
        WISP_CUDA_TRY(cudaFuncSetAttribute(down_gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes));
        attr_set[dev] = true;
    }
    CUtensorMap mx, mw13, mact, mw2;
    int rc = make_map(&mx, p.x_perm, (uint64_t)p.perm_rows, (uint64_t)p.H, kHalfN);
    if (!rc) rc = make_map(&mw13, p.w13, (uint64_t)p.slots * 2 * p.I, (uint64_t)p.H, kHalfN);
    if (!rc) rc = make_map(&mact, p.act_perm, (uint64_t)p.perm_rows, (uint64_t)p.I, kHalfN);
    if (!rc) rc = make_map(&mw2, p.w2, (uint64_t)p.slots * p.H, (uint64_t)p.I, kHalfN);
    if (rc) return rc;
    GroupGemm g{};
    g.u_off = p.u_off;
    g.u_pairs = p.u_pairs;
    g.u_slot = p.u_slot;
    g.nu_dev = p.nu_dev;
    g.pager_status = p.pager_status;
    g.H = p.H;
    g.I = p.I;
    g.K = p.K;
    g.topk_w = p.topk_w;
    g.act_perm = p.act_perm;
    g.y = p.y;
    g.status = p.status;
    g.wait_ns = p.wait_ns;
    // persistent grids: at most one CTA per SM (tiles: at most one partial
    // 128-pair tile per expert beyond the full ones; `nu` bounds the count)
    int sms = 0;
    WISP_CUDA_TRY(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
    const long mtiles = (long)p.nu + (p.npairs + kBM - 1) / kBM;
    const int grid_gu = (int)std::min<long>(mtiles * (p.I / kHalfN), sms);
    const int grid_dn = (int)std::min<long>(mtiles * (p.H / kBN), sms);
    if (gather) rc = launch_gather(p, stream);
    if (!rc)
        rc = launch_chained(gateup_gemm_kernel, dim3(grid_gu), dim3(kThreads), (size_t)kSmemBytes, stream, mx, mw13, g);
    if (!rc)
        rc = launch_chained(down_gemm_kernel, dim3(grid_dn), dim3(kThreads), (size_t)kSmemBytes, stream, mact, mw2, g);
    return rc ? rc : launch_combine(p, stream);
}

int launch_prefill_gemms(const PrefillGroup &p, cudaStream_t stream) { return launch_prefill_kernels(p, false, stream); }
}  // namespace

int launch_prefill_group(const PrefillGroup &p, cudaStream_t stream) { return launch_prefill_kernels(p, true, stream); }

int launch_prefill_resident(const PrefillGroup &p, const BatchRoute &r, const PrefillLists &lists,
                            cudaStream_t stream) {
    using namespace gemm;
    if (!prefill_shapes_supported(p.H, p.I))
        return set_error("wisp: prefill GEMM needs hidden % 256 == 0 and inter % 128 == 0"), WISP_ERR_UNSUPPORTED;
    if (p.npairs <= 0) return WISP_OK;
    if (r.E < 1 || r.E > kRouteMaxExperts)
        return set_error("wisp: resident routing takes at most 1024 experts"), WISP_ERR_INVALID;
    if (!lists.cnt || !lists.cnt_next || !lists.bar)
        return set_error("wisp: resident routing without its counters"), WISP_ERR_INVALID;
    int dev = 0, sms = 0;
    WISP_CUDA_TRY(cudaGetDevice(&dev));
    WISP_CUDA_TRY(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
    const int blocks = std::max(1, std::min(sms, (p.npairs + 63) / 64));
    const int per = (p.npairs + blocks - 1) / blocks;
    const size_t smem = sizeof(int2) * (size_t)per;
    if (smem > 160 * 1024) return set_error("wisp: resident call too large for one routing launch"), WISP_ERR_INVALID;
    static size_t smem_set[64] = {};
    if (dev < 0 || dev >= 64) return WISP_ERR_INVALID;
    if (smem_set[dev] < smem) {
        WISP_CUDA_TRY(cudaFuncSetAttribute(route_gather_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           (int)smem));
        smem_set[dev] = smem;
    }
    RouteArgs a{};
    a.ids = r.ids;
    a.ids64 = r.ids64;
    a.P = p.npairs;
    a.E = r.E;
    a.K = p.K;
    a.H8 = p.H / 8;
    a.count_forward = r.count_forward;
    a.emap = r.emap;
    a.x = reinterpret_cast<const uint4 *>(p.x);
    a.x_perm = reinterpret_cast<uint4 *>(p.x_perm);
    a.hdr = r.hdr;
    a.dev_hdr = r.dev_status;
    a.status = p.status;
    a.u_off = lists.u_off;
    a.u_pairs = lists.u_pairs;
    a.u_slot = lists.u_slot;
    a.nu = lists.nu;
    a.cnt = lists.cnt;
    a.cnt_next = lists.cnt_next;
    a.bar = lists.bar;
    a.wait_ns = p.wait_ns;
    int rc = launch_persistent(route_gather_kernel, dim3(blocks), dim3(kRouteThreads), smem, stream, a);
    return rc ? rc : launch_prefill_gemms(p, stream);
}

}  // namespace wisp
