// Prefill expert compute on the 5th-generation tensor cores (sm_100a):
// tcgen05.mma with the accumulator in tensor memory, operands staged in
// shared memory by TMA.  One token group of a forward, after its experts are
// resident in their slots:
//
//   gather      X_perm[q] = x[token of pair q], q in the group's expert-major
//               pair order (the pager's per-expert lists), so each expert's
//               tokens are consecutive rows;
//   gate-up     per expert u and tile of 128 of its pairs x 128 rows j of the
//               intermediate: D[128 x 256] = X_perm rows . [W13 gate rows j ;
//               up rows I + j]^T over K = H, so each thread of the epilogue
//               holds g and u of the same (pair, j) and stores
//               act_perm[q][j] = bf16(bf16(silu(bf16(g))) * bf16(u));
//   down        per expert u and tile of 128 pairs x 256 hidden rows h:
//               D = act_perm rows . W2 rows^T over K = I; the epilogue stores
//               y[pair][h] = bf16(D * routing weight);
//   combine     out[t] = sum over k in routing order of y[t*K + k] (combine_add, bf16).
//
// Kernel structure (persistent: at most one CTA of 6 warps per SM, each
// looping over output tiles in N-fastest order, so consecutive tiles share the
// token rows and one expert's weights stay in L2): warp 0 lane 0 issues the
// TMA loads of a 4-stage ring (A tile 128 x 64 and B tile 256 x 64 bf16 per
// stage, 128-byte swizzle, the canonical K-major layout of the MMA's
// shared-memory descriptors) continuously across tiles; warp 1 lane 0 issues
// tcgen05.mma (M 128, N 256, K 16) into one of two 256-column TMEM
// accumulators and commits each stage back to the producer's "empty" barrier
// and each finished accumulator to the epilogue; warps 2..5 read an
// accumulator back with tcgen05.ld (warp w owns TMEM lanes 32 (w % 4) ..,
// = tile rows) while the next tile accumulates into the other one.  Every
// wait is bounded by a %globaltimer limit; a wait that runs out records
// WISP_ERR_TIMEOUT in the status word, the roles stop, the CTA waits
// (bounded) for its copies and MMAs in flight, frees its tensor memory and
// returns.
//
// Per (pair, row) arithmetic is independent of which other pairs share a tile
// (each accumulator element is its own dot product, K blocks in order), so
// results do not depend on the grouping, the cap or the slots; they differ
// from the CUDA-core decode path only in the order of the fp32 accumulation.
#pragma once
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "common.cuh"
#include "prefill.cuh"

namespace wisp {
namespace gemm {

constexpr int kBM = 128;                       // pairs (tokens) per tile: TMEM lanes
constexpr int kBK = 64;                        // K per stage: one 128-byte swizzle row of bf16
constexpr int kBN = 256;                       // output columns per tile
constexpr int kHalfN = kBN / 2;                // one TMA box of B rows
constexpr int kStages = 4;
constexpr int kThreads = 192;                  // producer warp, MMA warp, 4 epilogue warps
constexpr int kEpiThreads = 128;
constexpr int kATileBytes = kBM * kBK * 2;     // 16 KB
constexpr int kBTileBytes = kBN * kBK * 2;     // 32 KB
constexpr int kStageBytes = kATileBytes + kBTileBytes;
constexpr int kSmemBytes = kStages * kStageBytes + 1024;  // + slack to align stages to 1024 B
constexpr int kAccCols = 256;                  // one accumulator
constexpr int kTmemCols = 2 * kAccCols;         // two, double-buffered

// Everything a group's GEMM kernels need besides the tensor maps.
struct GroupGemm {
    const int32_t *u_off;    // [nu + 1] pair-list offsets of the group's experts
    const int32_t *u_pairs;  // [P_g] absolute pair index (t * K + k), expert-major
    const int32_t *u_slot;   // [nu] slot of each expert
    const int32_t *nu_dev;   // experts in the group (device word written by the pager)
    const int32_t *pager_status;  // the pager's status word (nullptr: checked by the host)
    int H, I, K;             // hidden, intermediate, top-k
    const float *topk_w;     // [T * K] routing weights (absolute pair index)
    __nv_bfloat16 *act_perm; // [P_g][I] (gate-up output, down input)
    __nv_bfloat16 *y;        // [T * K][H] weighted rows (absolute pair index)
    int *status;             // sticky status word (first error wins)
    long long wait_ns;
};

// ---- PTX wrappers -------------------------------------------------------------
__device__ __forceinline__ uint32_t s_addr(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(s_addr(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(s_addr(bar)), "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ bool mbar_try(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}"
        : "=r"(ok)
        : "r"(s_addr(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}
// Bounded wait; false when it ran out (or `abort` was raised meanwhile).
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity, long long wait_ns,
                                          volatile int *abort) {
    if (mbar_try(bar, parity)) return true;
    const unsigned long long t0 = globaltimer_ns();
    while (!mbar_try(bar, parity)) {
        if (*abort) return false;
        if ((long long)(globaltimer_ns() - t0) > wait_ns) return false;
    }
    return true;
}
__device__ __forceinline__ void tma_load_2d(void *dst, const CUtensorMap *map, int x, int y, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::
            "r"(s_addr(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(s_addr(bar))
        : "memory");
}
__device__ __forceinline__ void tma_load_2d_hint(void *dst, const CUtensorMap *map, int x, int y, uint64_t *bar,
                                                 uint64_t policy) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1, {%2, "
        "%3}], [%4], %5;" ::"r"(s_addr(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(s_addr(bar)), "l"(policy)
        : "memory");
}
__device__ __forceinline__ uint64_t policy_evict_last() {
    uint64_t pol;
    asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(pol));
    return pol;
}
__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(s_addr(bar)) : "memory");
}
__device__ __forceinline__ void tmem_alloc(uint32_t *dst_smem, uint32_t cols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(s_addr(dst_smem)),
                 "r"(cols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t cols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(cols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
// D[tmem] (+)= A[smem] . B[smem]^T, M 128, N from the instruction descriptor, K 16.
__device__ __forceinline__ void umma_f16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                         uint32_t accumulate) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}" ::"r"(
            tmem_d),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}
// Arrive on `bar` once every MMA this thread issued so far has completed.
__device__ __forceinline__ void umma_commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(s_addr(bar))
                 : "memory");
}
// 32 lanes x 32 consecutive 32-bit columns of TMEM -> 32 registers per thread.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr)
        : "memory");
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// Shared-memory matrix descriptor of a K-major tile with 128-byte swizzle:
// rows of 64 bf16 (128 B), 8-row groups 1024 B apart (stride byte offset),
// start address in 16-byte units; descriptor version 1, layout type 2.
__device__ __forceinline__ uint64_t smem_desc_k_sw128(uint32_t saddr) {
    uint64_t d = 0;
    d |= (uint64_t)((saddr >> 4) & 0x3FFFu);          // start address
    d |= (uint64_t)1u << 16;                          // leading byte offset (unused with swizzle)
    d |= (uint64_t)(1024u >> 4) << 32;                // stride byte offset
    d |= (uint64_t)1u << 46;                          // version
    d |= (uint64_t)2u << 61;                          // SWIZZLE_128B
    return d;
}
// Instruction descriptor of kind::f16: bf16 A and B (K-major), fp32 D, M x N.
__host__ __device__ constexpr uint32_t idesc_bf16_f32(int M, int N) {
    return (1u << 4)                    // D format F32
           | (1u << 7)                  // A format BF16
           | (1u << 10)                 // B format BF16
           | ((uint32_t)(N >> 3) << 17) // N / 8
           | ((uint32_t)(M >> 4) << 24);// M / 16
}

// The status word is mapped host memory: a plain store (any non-zero code
// marks the failure; no atomics across PCIe).
__device__ __forceinline__ void record_timeout(const GroupGemm &g) {
    if (g.status) *reinterpret_cast<volatile int *>(g.status) = WISP_ERR_TIMEOUT;
}

// Shared state of a persistent GEMM CTA.
struct Ring {
    uint64_t full[kStages], empty[kStages];
    uint64_t acc_full[2], acc_empty[2], mma_done;
    uint32_t tmem_base;
    int abort;
    int issued, consumed;  // k-steps the producer filled / the MMA thread took
};

// A tile's operands: A rows [a_row, +128), B rows [b_row0, +128) and
// [b_row1, +128), K = kb_count * 64.
struct TileOperands {
    int a_row, b_row0, b_row1;
};

// Producer (warp 0 lane 0): fills the ring for every tile of this CTA.
template <class TileFn>
__device__ __forceinline__ void produce(const CUtensorMap *map_a, const CUtensorMap *map_b, int ntiles, int kb_count,
                                        unsigned char *stages, Ring &R, const GroupGemm &g, TileFn tile_operands) {
    volatile int *abort = &R.abort;
    const uint64_t keep = policy_evict_last();  // token rows: reused by the tile's other N columns
    int kstep = 0;
    for (int t = blockIdx.x; t < ntiles; t += gridDim.x) {
        const TileOperands op = tile_operands(t);
        for (int kb = 0; kb < kb_count; ++kb, ++kstep) {
            const int s = kstep % kStages;
            if (kstep >= kStages && !mbar_wait(&R.empty[s], ((kstep / kStages) - 1) & 1, g.wait_ns, abort)) {
                R.abort = 1;
                record_timeout(g);
                return;
            }
            unsigned char *st = stages + s * kStageBytes;
            mbar_expect_tx(&R.full[s], kStageBytes);
            tma_load_2d_hint(st, map_a, kb * kBK, op.a_row, &R.full[s], keep);
            tma_load_2d(st + kATileBytes, map_b, kb * kBK, op.b_row0, &R.full[s]);
            tma_load_2d(st + kATileBytes + kHalfN * kBK * 2, map_b, kb * kBK, op.b_row1, &R.full[s]);
            R.issued = kstep + 1;
        }
    }
}

// MMA issuer (warp 1 lane 0): accumulates tile i into accumulator i % 2.
__device__ __forceinline__ void issue_mmas(int ntiles, int kb_count, unsigned char *stages, Ring &R,
                                           const GroupGemm &g) {
    volatile int *abort = &R.abort;
    const uint32_t idesc = idesc_bf16_f32(kBM, kBN);
    int kstep = 0, i = 0;
    for (int t = blockIdx.x; t < ntiles; t += gridDim.x, ++i) {
        const int b = i & 1;
        if (i >= 2 && !mbar_wait(&R.acc_empty[b], ((i / 2) - 1) & 1, g.wait_ns, abort)) {
            R.abort = 1;
            record_timeout(g);
            break;
        }
        tc_fence_after();
        const uint32_t acc = R.tmem_base + b * kAccCols;
        bool ok = true;
        for (int kb = 0; kb < kb_count; ++kb, ++kstep) {
            const int s = kstep % kStages;
            if (!mbar_wait(&R.full[s], (kstep / kStages) & 1, g.wait_ns, abort)) {
                R.abort = 1;
                record_timeout(g);
                ok = false;
                break;
            }
            tc_fence_after();
            const uint32_t a0 = s_addr(stages + s * kStageBytes), b0 = a0 + kATileBytes;
#pragma unroll
            for (int kk = 0; kk < kBK / 16; ++kk)  // 16 bf16 = 32 bytes further along K
                umma_f16(acc, smem_desc_k_sw128(a0 + kk * 32), smem_desc_k_sw128(b0 + kk * 32), idesc,
                         (kb | kk) != 0);
            umma_commit(&R.empty[s]);
            R.consumed = kstep + 1;
        }
        if (!ok) break;
        umma_commit(&R.acc_full[b]);
    }
    umma_commit(&R.mma_done);  // every MMA issued (also after an abort)
}

// After an abort (all threads past the roles): wait, bounded, for the copies
// issued but not taken by the MMA thread and for the MMAs issued, so none
// outlives the CTA.
__device__ __forceinline__ void drain_ring(Ring &R, const GroupGemm &g) {
    if (threadIdx.x != 0) return;
    volatile int no_abort = 0;
    for (int k = R.consumed; k < R.issued; ++k)
        mbar_wait(&R.full[k % kStages], (k / kStages) & 1, g.wait_ns, &no_abort);
    mbar_wait(&R.mma_done, 0, g.wait_ns, &no_abort);
}

// Experts of the group as the kernels see them: the pager's count, or none
// when the pager (run on the device without a host check) rejected the call.
__device__ __forceinline__ int group_experts(const int32_t *nu_dev, const int32_t *pager_status) {
    if (pager_status && *reinterpret_cast<const volatile int32_t *>(pager_status) != WISP_OK) return 0;
    return *reinterpret_cast<const volatile int32_t *>(nu_dev);
}

// ---- host helpers shared by the token-major and weight-stationary paths ------------
// Row-major bf16 matrix [rows][cols] (16-byte aligned base, cols % 8 == 0) as
// 64 x box_rows boxes with 128-byte swizzle.
int make_map(CUtensorMap *map, const void *base, uint64_t rows, uint64_t cols, uint32_t box_rows);
// X_perm rows of the group.
int launch_gather(const PrefillGroup &p, cudaStream_t stream);
// out rows [t0, t1) = routing-order sum of the weighted rows y.
int launch_combine(const PrefillGroup &p, cudaStream_t stream);

}  // namespace gemm
}  // namespace wisp
