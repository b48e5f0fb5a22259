// Shared helpers for the wisp_b200 kernels and runtime (sm_100a only).
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <string>

#include "../../include/wisp_b200.h"

#if defined(__CUDA_ARCH__) && (__CUDA_ARCH__ < 1000)
#error "wisp_b200 kernels are written for sm_100a (B200) only"
#endif

namespace wisp {

// Thread-local message of the last failing C-ABI call.
void set_error(const std::string &msg);

#define WISP_CUDA_TRY(expr)                                                          \
    do {                                                                             \
        cudaError_t _e = (expr);                                                     \
        if (_e != cudaSuccess) {                                                     \
            ::wisp::set_error(std::string(#expr) + ": " + cudaGetErrorString(_e));   \
            return WISP_ERR_CUDA;                                                    \
        }                                                                            \
    } while (0)

// Cooperative launch of a persistent kernel (every block resident: blocks wait
// on one another), with programmatic dependent launch when WISP_PDL is set:
// the launch may begin while the previous kernel on the stream drains,
// and the kernel's pdl_wait() orders it after that kernel.  If the driver
// refuses the two attributes together, the plain cooperative launch is used
// from then on for that device.
bool pdl_enabled(int dev);
void pdl_refused(int dev);
template <typename... KArgs, typename... Args>
int launch_persistent(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                      Args... args) {
    int dev = 0;
    WISP_CUDA_TRY(cudaGetDevice(&dev));
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    if (pdl_enabled(dev)) {
        cfg.numAttrs = 2;
        if (cudaLaunchKernelEx(&cfg, kernel, args...) == cudaSuccess) return WISP_OK;
        (void)cudaGetLastError();  // a refused launch configuration, not a device fault
        pdl_refused(dev);
    }
    cfg.numAttrs = 1;
    WISP_CUDA_TRY(cudaLaunchKernelEx(&cfg, kernel, args...));
    return WISP_OK;
}

// The same for a kernel whose blocks do not wait on one another (no
// cooperative launch), still with programmatic dependent launch.
template <typename... KArgs, typename... Args>
int launch_chained(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                   Args... args) {
    int dev = 0;
    WISP_CUDA_TRY(cudaGetDevice(&dev));
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    if (pdl_enabled(dev)) {
        cfg.numAttrs = 1;
        if (cudaLaunchKernelEx(&cfg, kernel, args...) == cudaSuccess) return WISP_OK;
        (void)cudaGetLastError();
        pdl_refused(dev);
    }
    cfg.numAttrs = 0;
    WISP_CUDA_TRY(cudaLaunchKernelEx(&cfg, kernel, args...));
    return WISP_OK;
}

// ---- bf16 helpers -------------------------------------------------------
__device__ __forceinline__ float bf16lo(uint32_t v) { return __uint_as_float(v << 16); }
__device__ __forceinline__ float bf16hi(uint32_t v) { return __uint_as_float(v & 0xffff0000u); }
__device__ __forceinline__ float round_bf16(float v) {
    return __bfloat162float(__float2bfloat16_rn(v));
}

// 8 bf16 (one 16-byte vector) dotted with 8 bf16, fp32 FMA chain in element order.
// acc += w[0]*x[0] + ... + w[7]*x[7] as an FMA chain in element order (low
// half of each 32-bit word first).  fma.rn.f32.bf16 multiplies the bf16
// operands exactly (an 8-bit x 8-bit significand product fits in fp32) and
// rounds once, so each step equals fmaf on the operands widened to fp32; it
// needs no widening instructions.
__device__ __forceinline__ float fma2_bf16(uint32_t w, uint32_t x, float acc) {
    asm("{\n .reg .b16 wl, wh, xl, xh;\n mov.b32 {wl, wh}, %1;\n mov.b32 {xl, xh}, %2;\n"
        " fma.rn.f32.bf16 %0, wl, xl, %0;\n fma.rn.f32.bf16 %0, wh, xh, %0;\n}"
        : "+f"(acc)
        : "r"(w), "r"(x));
    return acc;
}
__device__ __forceinline__ float dot8(const uint4 &w, const uint4 &x, float acc) {
    acc = fma2_bf16(w.x, x.x, acc);
    acc = fma2_bf16(w.y, x.y, acc);
    acc = fma2_bf16(w.z, x.z, acc);
    acc = fma2_bf16(w.w, x.w, acc);
    return acc;
}

// Activation element as stored.  The all-ones bf16 pattern (a NaN) marks an
// element the one-launch forward has not written yet, so a result with that
// pattern is stored as the canonical NaN instead (every path does the same).
constexpr unsigned short kActEmpty = 0xFFFFu;
// The reference's storage points around the activation and the combine
// (vLLM's silu_and_mul and moe_sum, pinned by golden outputs of vLLM's
// fused_experts): silu(g) is stored bf16 before it multiplies u, and the k
// weighted rows of a token are added in bf16 -- every partial sum rounded --
// for top-k <= 4, in fp32 above.
__device__ __forceinline__ float silu_stored(float g) { return round_bf16(g / (1.0f + expf(-g))); }
__device__ __forceinline__ float combine_add(float acc, float v, int K) {
    return K <= 4 ? round_bf16(acc + v) : acc + v;
}

__device__ __forceinline__ __nv_bfloat16 act_value(float v) {
    __nv_bfloat16 b = __float2bfloat16_rn(v);
    if (__bfloat16_as_ushort(b) == kActEmpty) b = __ushort_as_bfloat16((unsigned short)0x7FFFu);
    return b;
}
// A 2-byte store other SMs poll for (relaxed, device scope: no data race).
__device__ __forceinline__ void st_relaxed_bf16(__nv_bfloat16 *p, __nv_bfloat16 v) {
    asm volatile("st.relaxed.gpu.global.b16 [%0], %1;" ::"l"(p), "h"(__bfloat16_as_ushort(v)) : "memory");
}
// 16-byte load that always reads the coherent level (polling other SMs' stores).
__device__ __forceinline__ uint4 ld_volatile16(const void *p) {
    uint4 r;
    asm volatile("ld.volatile.global.v4.u32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "l"(p)
                 : "memory");
    return r;
}
__device__ __forceinline__ bool half_empty(uint32_t w) {
    return (w & 0xFFFFu) == kActEmpty || (w >> 16) == kActEmpty;
}
// Any of the eight bf16 elements still the "not written" pattern?
__device__ __forceinline__ bool has_empty(const uint4 &v) {
    return half_empty(v.x) | half_empty(v.y) | half_empty(v.z) | half_empty(v.w);
}

// Streaming 16-byte load for weights read once per forward (no L1 allocation).
__device__ __forceinline__ uint4 ld_stream16(const void *p) {
    uint4 r;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "l"(p));
    return r;
}

__device__ __forceinline__ uint4 ld_cached16(const void *p) {
    return __ldg(reinterpret_cast<const uint4 *>(p));
}

// Coherent 16-byte load cached in L2 only: for data written during the same
// kernel (by other CTAs or by the copy engine), which the non-coherent
// read-only path must not serve.
__device__ __forceinline__ uint4 ld_cg16(const void *p) {
    return __ldcg(reinterpret_cast<const uint4 *>(p));
}

__device__ __forceinline__ unsigned long long globaltimer_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// Programmatic dependent launch.  A kernel launched with the programmatic
// stream-serialization attribute may start while the kernel before it on the
// stream still runs; pdl_wait() returns once that kernel has completed and
// its memory is visible, so every read or write of device memory that other
// work produced or consumes comes after it.  pdl_launch_dependents() lets the
// next such kernel start (its blocks then occupy SMs this kernel's blocks
// have left and wait there).  Both are no-ops for a plain launch.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// Butterfly sum over the warp; every lane ends with the same value and the
// pairing order is fixed, so the result is independent of anything but the
// 32 inputs.
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// Routed expert id i of an int32 or int64 id array (range-checked by callers).
__device__ __forceinline__ long long load_id64(const void *ids, int ids64, long i) {
    return ids64 ? reinterpret_cast<const long long *>(ids)[i]
                 : (long long)reinterpret_cast<const int *>(ids)[i];
}

}  // namespace wisp
