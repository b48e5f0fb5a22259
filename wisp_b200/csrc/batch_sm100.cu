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
//            bf16(silu(bf16(g)) * bf16(u));
//   down     tile (token block b, 256 hidden rows h):
//            Y0 / Y1 [128 x 32] = W2 rows h / h + 128 . act_perm rows^T over
//            K = I; y[pair][h + r] = bf16(acc * routing weight).
//
// A token block is up to 32 consecutive rows of one expert in the group's
// expert-major pair order (X_perm, written by the gather kernel), so each
// weight tile is streamed once per token block, i.e. once per expert for a
// decode batch.  Gate-up and down share ONE persistent launch: tiles are
// numbered gate-up first, then down, both in token-block order, and each CTA
// walks its tiles (t = blockIdx.x, + gridDim.x, ...) in that order.  Before
// the producer loads a down tile it waits until the block's gate-up tiles
// have published their activation rows: every epilogue warp adds 1 to the
// block's counter after its stores (release at GPU scope, after an
// async-proxy fence, since the rows are read back by TMA), and the producer
// waits for 4 * I / 128 (acquire, then an async-proxy fence).  Gate-up tiles
// wait for nothing, and the launch is cooperative (every CTA resident), so
// these waits end; each is bounded all the same and a CTA that gives up
// raises a device-wide abort word that ends the others' waits.
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
// the cap or the grouping.
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
constexpr int kMaxExperts = 1024;
static_assert(kTmemCols >= 32 && (kTmemCols & (kTmemCols - 1)) == 0, "TMEM allocation: power of two >= 32");
static_assert(kTN % 16 == 0 && kTN >= 16 && kTN <= 256, "MMA N for M = 128");

struct Args {
    const int32_t *u_off;     // [nu + 1]
    const int32_t *u_pairs;   // [npairs] absolute pair index, expert-major
    const int32_t *u_slot;    // [nu]
    const int32_t *nu_dev;
    const int32_t *pager_status;
    int H, I;
    const float *topk_w;      // [T * K]
    __nv_bfloat16 *act_perm;  // [npairs][I]
    __nv_bfloat16 *y;         // [T * K][H]
    uint32_t *ready;          // [blocks] gate-up warps done per token block; [nready - 1] abort word
    int nready;
    int *status;
    long long wait_ns;
};

struct Ring {
    uint64_t full[kStages], empty[kStages];
    uint64_t acc_full[2], acc_empty[2], mma_done;
    uint32_t tmem_base;
    int abort;
    int issued, consumed;
};

struct BlockTable {
    int nu, nblocks;
    int off[kMaxExperts + 1];    // pair-list offsets
    int first[kMaxExperts + 1];  // first token block of each expert (prefix of block counts)
};

// Token block b -> expert u, first list position q0, rows.
__device__ __forceinline__ void block_of(const BlockTable &bt, int b, int &u, int &q0, int &rows) {
    int lo = 0, hi = bt.nu - 1;
    while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (bt.first[mid] <= b)
            lo = mid;
        else
            hi = mid - 1;
    }
    u = lo;
    q0 = bt.off[u] + (b - bt.first[u]) * kTN;
    rows = min(kTN, bt.off[u + 1] - q0);
}

struct Tile {
    int down;  // 0: gate-up, 1: down
    int b;     // token block
    int col;   // 128-row block of I (gate-up) or 256-row block of H (down)
};
__device__ __forceinline__ Tile tile_at(int t, int ngu, int cj, int ch) {
    if (t < ngu) return Tile{0, t / cj, t % cj};
    t -= ngu;
    return Tile{1, t / ch, t % ch};
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

__device__ __forceinline__ void give_up(Ring &R, const Args &g) {
    R.abort = 1;
    if (g.status) *reinterpret_cast<volatile int *>(g.status) = WISP_ERR_TIMEOUT;
    atomicExch(g.ready + g.nready - 1, 1u);  // ends the other CTAs' waits
}

// Producer wait for a down tile: the block's activation rows are published.
__device__ __forceinline__ bool wait_ready(const Args &g, int b, uint32_t need, volatile int *abort) {
    const uint32_t *word = g.ready + b;
    const volatile uint32_t *abort_all = g.ready + g.nready - 1;
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

__device__ __forceinline__ unsigned char *align1024(unsigned char *p) {
    const uint32_t a = s_addr(p);
    return p + ((1024u - (a & 1023u)) & 1023u);
}

__global__ void __launch_bounds__(kThreads, 1)
    batch_moe_kernel(const __grid_constant__ CUtensorMap map_w13, const __grid_constant__ CUtensorMap map_w2,
                     const __grid_constant__ CUtensorMap map_x, const __grid_constant__ CUtensorMap map_act,
                     const Args g) {
    extern __shared__ unsigned char smem_raw[];
    __shared__ Ring R;
    __shared__ BlockTable bt;
    unsigned char *stages = align1024(smem_raw);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    // ---- setup: block table, barriers, TMEM ----------------------------------------
    const int nu = min(gemm::group_experts(g.nu_dev, g.pager_status), kMaxExperts);
    for (int i = threadIdx.x; i <= nu; i += blockDim.x) bt.off[i] = g.u_off[i];
    __syncthreads();
    if (threadIdx.x == 0) {
        bt.nu = nu;
        int acc = 0;
        for (int e = 0; e < nu; ++e) {
            bt.first[e] = acc;
            acc += (bt.off[e + 1] - bt.off[e] + kTN - 1) / kTN;
        }
        bt.first[nu] = acc;
        bt.nblocks = acc;
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
    const int H = g.H, I = g.I;
    const int cj = I / kWM, ch = H / kDownRows;
    const int ngu = bt.nblocks * cj;
    const int ntiles = ngu + bt.nblocks * ch;
    if ((int)blockIdx.x >= ntiles) return;
    if (warp == 0) tmem_alloc(&R.tmem_base, kTmemCols);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    volatile int *abort = &R.abort;
    const uint32_t need = (uint32_t)(kEpiWarps * cj);

    if (warp == 0) {
        // ---- producer --------------------------------------------------------------
        if (lane == 0) {
            const uint64_t once = policy_evict_first();  // each weight tile is read once
            int kstep = 0;
            for (int t = blockIdx.x; t < ntiles; t += gridDim.x) {
                const Tile tl = tile_at(t, ngu, cj, ch);
                int u, q0, rows;
                block_of(bt, tl.b, u, q0, rows);
                const int slot = g.u_slot[u];
                const CUtensorMap *mw, *mt;
                int a0, a1, kbc;
                if (!tl.down) {
                    mw = &map_w13;
                    mt = &map_x;
                    a0 = slot * 2 * I + tl.col * kWM;
                    a1 = a0 + I;
                    kbc = H / kBK;
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
                for (int kb = 0; kb < kbc; ++kb, ++kstep) {
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
                    R.issued = kstep + 1;
                }
                if (!ok) {
                    give_up(R, g);
                    break;
                }
            }
        }
    } else if (warp == 1) {
        // ---- MMA issuer -------------------------------------------------------------
        if (lane == 0) {
            const uint32_t idesc = gemm::idesc_bf16_f32(kWM, kTN);
            int kstep = 0, i = 0;
            for (int t = blockIdx.x; t < ntiles; t += gridDim.x, ++i) {
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
        }
    } else {
        // ---- epilogue (warps 2..5) ----------------------------------------------------
        const int quarter = warp & 3, r = quarter * 32 + lane;
        int i = 0;
        for (int t = blockIdx.x; t < ntiles; t += gridDim.x, ++i) {
            const bool ok = mbar_wait(&R.acc_full[i & 1], (i / 2) & 1, g.wait_ns, abort) && !*abort;
            if (!__all_sync(0xffffffffu, ok)) break;  // uniform: the TMEM loads are .sync.aligned
            tc_fence_after();
            const Tile tl = tile_at(t, ngu, cj, ch);
            int u, q0, rows;
            block_of(bt, tl.b, u, q0, rows);
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
                        dst[(size_t)n * I] = act_value(gv / (1.0f + expf(-gv)) * uv);
                    }
                }
                fence_proxy_async_global();
                __syncwarp();
                if (lane == 0) {
                    __threadfence();
                    red_release_gpu_add(g.ready + tl.b, 1u);
                }
            } else {
                const int h = tl.col * kDownRows + r;
#pragma unroll
                for (int n = 0; n < kTN; ++n) {
                    if (n < rows) {
                        const int p = g.u_pairs[q0 + n];
                        const float wp = g.topk_w[p];
                        __nv_bfloat16 *dst = g.y + (size_t)p * H + h;
                        dst[0] = __float2bfloat16_rn(__uint_as_float(d0[n]) * wp);
                        dst[kWM] = __float2bfloat16_rn(__uint_as_float(d1[n]) * wp);
                    }
                }
            }
        }
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
}

}  // namespace
}  // namespace batch

int launch_batch_group(const PrefillGroup &p, cudaStream_t stream) {
    using namespace batch;
    if (!prefill_shapes_supported(p.H, p.I))
        return set_error("wisp: tensor-core path needs hidden % 256 == 0 and inter % 128 == 0"), WISP_ERR_UNSUPPORTED;
    if (p.npairs <= 0 || p.nu <= 0) return WISP_OK;
    if (!p.ready) return set_error("wisp: batch path without its counter workspace"), WISP_ERR_INVALID;
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
    Args a{};
    a.u_off = p.u_off;
    a.u_pairs = p.u_pairs;
    a.u_slot = p.u_slot;
    a.nu_dev = p.nu_dev;
    a.pager_status = p.pager_status;
    a.H = p.H;
    a.I = p.I;
    a.topk_w = p.topk_w;
    a.act_perm = p.act_perm;
    a.y = p.y;
    a.ready = p.ready;
    a.nready = (int)batch_ready_words(p.npairs, p.nu);
    a.status = p.status;
    a.wait_ns = p.wait_ns;
    rc = gemm::launch_gather(p, a.ready, a.nready, stream);
    if (rc) return rc;
    // persistent and cooperative: at most one CTA per SM, all resident (the
    // down tiles wait for gate-up tiles of other CTAs)
    int sms = 0;
    WISP_CUDA_TRY(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
    const long blocks = std::min<long>(p.nu, p.npairs) + (p.npairs + kTN - 1) / kTN;
    const long tiles = blocks * (p.I / kWM + p.H / kDownRows);
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3((unsigned)std::min<long>(tiles, sms));
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = kSmemBytes;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    WISP_CUDA_TRY(cudaLaunchKernelEx(&cfg, batch_moe_kernel, mw13, mw2, mx, mact, a));
    return gemm::launch_combine(p, stream);
}

}  // namespace wisp
