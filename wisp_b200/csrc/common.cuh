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

// ---- bf16 helpers -------------------------------------------------------
__device__ __forceinline__ float bf16lo(uint32_t v) { return __uint_as_float(v << 16); }
__device__ __forceinline__ float bf16hi(uint32_t v) { return __uint_as_float(v & 0xffff0000u); }
__device__ __forceinline__ float round_bf16(float v) {
    return __bfloat162float(__float2bfloat16_rn(v));
}

// 8 bf16 (one 16-byte vector) dotted with 8 bf16, fp32 FMA chain in element order.
__device__ __forceinline__ float dot8(const uint4 &w, const uint4 &x, float acc) {
    acc = fmaf(bf16lo(w.x), bf16lo(x.x), acc);
    acc = fmaf(bf16hi(w.x), bf16hi(x.x), acc);
    acc = fmaf(bf16lo(w.y), bf16lo(x.y), acc);
    acc = fmaf(bf16hi(w.y), bf16hi(x.y), acc);
    acc = fmaf(bf16lo(w.z), bf16lo(x.z), acc);
    acc = fmaf(bf16hi(w.z), bf16hi(x.z), acc);
    acc = fmaf(bf16lo(w.w), bf16lo(x.w), acc);
    acc = fmaf(bf16hi(w.w), bf16hi(x.w), acc);
    return acc;
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
