// K3: per-group expert compute from the slot scratch (memory-bound GEMV),
// used by the host-synchronous forward and by the allocation-free entry
// point.  The arithmetic lives in moe_body.cuh (shared with forward.cu).
//
// gateup_silu_kernel: grid (ceil(I/8), max_nu); warp w of block (bx, u)
//   handles row pair (j, I+j), j = 8*bx + w, of unique expert u for all of
//   u's pairs; each weight row is read once (streamed).
// down_combine_kernel: grid (ceil(H/8), max_nu); warp w handles row h of
//   W2[u] for all of u's pairs and stores the weighted y.  The last CTA to
//   finish a row block (arrival counter) sums the group's tokens over k in
//   routing order for those 8 rows and writes out.
#include "moe_body.cuh"

namespace wisp {

namespace {

constexpr int kWarps = 8;
constexpr int kRowsPerBlock = kWarps;

template <int MAXP>
__global__ void __launch_bounds__(kWarps * 32) gateup_silu_kernel(GroupCompute a) {
    const int u = blockIdx.y;
    if (u >= *a.nu) return;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int j = blockIdx.x * kRowsPerBlock + warp;
    if (j >= a.I) return;
    gateup_rowpair<MAXP>(a, u, j, lane);
}

template <int MAXP>
__global__ void __launch_bounds__(kWarps * 32) down_combine_kernel(GroupCompute a) {
    __shared__ int s_last;
    const int u = blockIdx.y;
    const int nu = *a.nu;
    if (u >= nu) return;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int h = blockIdx.x * kRowsPerBlock + warp;
    if (h < a.H) down_row<MAXP>(a, u, h, lane);
    // arrival: the last of the nu CTAs of this row block does the combine
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) s_last = (atomicAdd(&a.counters[blockIdx.x], 1) == nu - 1);
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    combine_rows(a, blockIdx.x * kRowsPerBlock, kRowsPerBlock, threadIdx.x, blockDim.x);
    if (threadIdx.x == 0) a.counters[blockIdx.x] = 0;
}

template <int MAXP>
int launch_variant(const GroupCompute &g, int max_nu, cudaStream_t stream) {
    dim3 block(kWarps * 32);
    dim3 g1((g.I + kRowsPerBlock - 1) / kRowsPerBlock, max_nu);
    gateup_silu_kernel<MAXP><<<g1, block, 0, stream>>>(g);
    WISP_CUDA_TRY(cudaGetLastError());
    dim3 g2((g.H + kRowsPerBlock - 1) / kRowsPerBlock, max_nu);
    down_combine_kernel<MAXP><<<g2, block, 0, stream>>>(g);
    WISP_CUDA_TRY(cudaGetLastError());
    return WISP_OK;
}

template <int MAXP>
cudaError_t preload_variant() {
    cudaFuncAttributes fa;
    cudaError_t e = cudaFuncGetAttributes(&fa, gateup_silu_kernel<MAXP>);
    if (e == cudaSuccess) e = cudaFuncGetAttributes(&fa, down_combine_kernel<MAXP>);
    return e;
}

}  // namespace

int preload_decode_kernels() {
    for (cudaError_t e : {preload_variant<1>(), preload_variant<2>(), preload_variant<4>(),
                          preload_variant<8>(), preload_variant<16>()})
        WISP_CUDA_TRY(e);
    return WISP_OK;
}

int launch_decode_group(const GroupCompute &g, int max_nu, cudaStream_t stream) {
    if (max_nu <= 0 || g.t1 <= g.t0) return WISP_OK;
    const int ntok = g.t1 - g.t0;
    if (ntok <= 1) return launch_variant<1>(g, max_nu, stream);
    if (ntok <= 2) return launch_variant<2>(g, max_nu, stream);
    if (ntok <= 4) return launch_variant<4>(g, max_nu, stream);
    if (ntok <= 8) return launch_variant<8>(g, max_nu, stream);
    return launch_variant<16>(g, max_nu, stream);
}

}  // namespace wisp
