// Per-layer runtime behind the C ABI (include/wisp_b200.h).
//
// A wisp_layer is the B200 counterpart of the reference's WispMoEState
// (src/wisp/integrations/vllm/fused_moe.py:126-490): slot scratch in HBM,
// the expert map and LRU state in device memory (updated by the device
// pager, K1), a copy-engine stream for page-in from the caller's pinned host
// masters, and the compute kernels (K3).
//
// Forward (wisp_moe_forward), per call:
//   1. K1 on the caller's stream: groups + LRU for every group, page-in list
//      into a mapped pinned mailbox;
//   2. the host waits for K1 (one event), reads the mailbox;
//   3. per group g: the group's page-ins go to the copy stream after the
//      compute event of the last earlier group of this call that read the
//      victim slot (write-after-read); the caller's stream waits for the
//      copies, then runs K3 for the group and records the group's event.
// Copies of one group overlap the compute of earlier groups whenever the
// victims were not read by them.
#include <algorithm>
#include <mutex>
#include <string>
#include <vector>

#include "common.cuh"
#include "decode.cuh"
#include "pager.cuh"

namespace wisp {

static thread_local std::string g_last_error;
void set_error(const std::string &msg) { g_last_error = msg; }

namespace {

struct DeviceGuard {
    int prev = -1;
    explicit DeviceGuard(int dev) {
        if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
        if (prev != dev) cudaSetDevice(dev);
    }
    ~DeviceGuard() {
        int cur = -1;
        if (prev >= 0 && cudaGetDevice(&cur) == cudaSuccess && cur != prev) cudaSetDevice(prev);
    }
};

int fail(int code, const std::string &msg) {
    set_error(msg);
    return code;
}

bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

__global__ void fill_identity_kernel(int32_t *s2e, int32_t *emap, int n) {
    int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) {
        s2e[i] = i;
        emap[i] = i;
    }
}

}  // namespace
}  // namespace wisp

using namespace wisp;

struct wisp_layer {
    int dev = 0, E = 0, cap = 0, H = 0, I = 0, mode = WISP_MODE_PAGED;
    int64_t b13 = 0, b2 = 0;
    const char *h13 = nullptr, *h2 = nullptr;
    char *d13 = nullptr, *d2 = nullptr;
    int32_t *d_s2e = nullptr, *d_emap = nullptr;
    int64_t *d_tick = nullptr, *d_hdr = nullptr;
    // per-call workspace, grown on demand
    int wsT = -1, wsK = 0;
    int32_t *d_slots = nullptr, *d_grp_start = nullptr, *d_grp_nu = nullptr, *d_u_slot = nullptr,
            *d_u_off = nullptr, *d_u_pairs = nullptr, *d_counters = nullptr;
    __nv_bfloat16 *d_act = nullptr, *d_y = nullptr;
    int32_t *h_mb = nullptr, *d_mb = nullptr;
    long mb_words = 0;
    cudaStream_t copy_stream = nullptr;
    cudaEvent_t ev_pager = nullptr, ev_copies = nullptr;
    std::vector<cudaEvent_t> ev_group, ev_copy;
    int64_t info[4] = {0, 0, 0, 0};
    std::mutex mu;
};

namespace {

void free_ws(wisp_layer *L) {
    cudaFree(L->d_slots);
    cudaFree(L->d_grp_start);
    cudaFree(L->d_grp_nu);
    cudaFree(L->d_u_slot);
    cudaFree(L->d_u_off);
    cudaFree(L->d_u_pairs);
    cudaFree(L->d_counters);
    cudaFree(L->d_act);
    cudaFree(L->d_y);
    if (L->h_mb) cudaFreeHost(L->h_mb);
    L->d_slots = L->d_grp_start = L->d_grp_nu = L->d_u_slot = L->d_u_off = L->d_u_pairs =
        L->d_counters = nullptr;
    L->d_act = L->d_y = nullptr;
    L->h_mb = L->d_mb = nullptr;
    L->wsT = -1;
    L->wsK = 0;
}

int ensure_ws(wisp_layer *L, int T, int K) {
    if (T <= L->wsT && K <= L->wsK) return WISP_OK;
    int nT = std::max(T, std::max(L->wsT, 16)), nK = std::max(K, L->wsK);
    free_ws(L);
    const size_t P = (size_t)nT * nK;
    WISP_CUDA_TRY(cudaMalloc(&L->d_slots, sizeof(int32_t) * std::max<size_t>(P, 1)));
    WISP_CUDA_TRY(cudaMalloc(&L->d_grp_start, sizeof(int32_t) * (nT + 1)));
    WISP_CUDA_TRY(cudaMalloc(&L->d_grp_nu, sizeof(int32_t) * (nT + 1)));
    WISP_CUDA_TRY(cudaMalloc(&L->d_u_slot, sizeof(int32_t) * std::max<size_t>(P, 1)));
    WISP_CUDA_TRY(cudaMalloc(&L->d_u_off, sizeof(int32_t) * (P + nT + 1)));
    WISP_CUDA_TRY(cudaMalloc(&L->d_u_pairs, sizeof(int32_t) * std::max<size_t>(P, 1)));
    const int H = std::max(L->H, 8), I = std::max(L->I, 8);
    const int nblk = (H + 7) / 8;
    WISP_CUDA_TRY(cudaMalloc(&L->d_counters, sizeof(int32_t) * nblk));
    WISP_CUDA_TRY(cudaMemset(L->d_counters, 0, sizeof(int32_t) * nblk));
    if (L->H > 0 && L->I > 0) {
        WISP_CUDA_TRY(cudaMalloc(&L->d_act, sizeof(__nv_bfloat16) * std::max<size_t>(P, 1) * I));
        WISP_CUDA_TRY(cudaMalloc(&L->d_y, sizeof(__nv_bfloat16) * std::max<size_t>(P, 1) * H));
    }
    L->mb_words = mailbox_words(nT, nK);
    WISP_CUDA_TRY(cudaHostAlloc(&L->h_mb, sizeof(int32_t) * L->mb_words, cudaHostAllocMapped));
    WISP_CUDA_TRY(cudaHostGetDevicePointer((void **)&L->d_mb, L->h_mb, 0));
    L->wsT = nT;
    L->wsK = nK;
    return WISP_OK;
}

int ensure_events(wisp_layer *L, int G) {
    while ((int)L->ev_group.size() < G) {
        cudaEvent_t a, b;
        WISP_CUDA_TRY(cudaEventCreateWithFlags(&a, cudaEventDisableTiming));
        WISP_CUDA_TRY(cudaEventCreateWithFlags(&b, cudaEventDisableTiming));
        L->ev_group.push_back(a);
        L->ev_copy.push_back(b);
    }
    return WISP_OK;
}

int alloc_state(wisp_layer *L, int cap) {
    WISP_CUDA_TRY(cudaMalloc(&L->d13, (size_t)cap * L->b13));
    WISP_CUDA_TRY(cudaMalloc(&L->d2, (size_t)cap * L->b2));
    WISP_CUDA_TRY(cudaMalloc(&L->d_s2e, sizeof(int32_t) * cap));
    WISP_CUDA_TRY(cudaMalloc(&L->d_tick, sizeof(int64_t) * cap));
    WISP_CUDA_TRY(cudaMemset(L->d_s2e, 0xff, sizeof(int32_t) * cap));
    WISP_CUDA_TRY(cudaMemset(L->d_tick, 0, sizeof(int64_t) * cap));
    return WISP_OK;
}

// Run K1 and wait for it; returns the pager status.
int run_pager(wisp_layer *L, const void *ids, int ids64, int T, int K, int single_group,
              int count_forward, cudaStream_t stream) {
    int rc = ensure_ws(L, T, K);
    if (rc) return rc;
    PagerParams p{};
    p.ids = ids;
    p.ids64 = ids64;
    p.T = T;
    p.K = K;
    p.E = L->E;
    p.cap = L->cap;
    p.mode = L->mode;
    p.count_forward = count_forward;
    p.single_group = single_group;
    p.s2e = L->d_s2e;
    p.tick = L->d_tick;
    p.emap = L->d_emap;
    p.hdr = L->d_hdr;
    p.slots = L->d_slots;
    p.grp_start = L->d_grp_start;
    p.grp_nu = L->d_grp_nu;
    p.u_slot = L->d_u_slot;
    p.u_off = L->d_u_off;
    p.u_pairs = L->d_u_pairs;
    p.mb = L->d_mb;
    L->h_mb[0] = -1;
    WISP_CUDA_TRY(cudaStreamWaitEvent(stream, L->ev_copies, 0));
    rc = launch_pager(p, stream);
    if (rc) return rc;
    WISP_CUDA_TRY(cudaEventRecord(L->ev_pager, stream));
    WISP_CUDA_TRY(cudaEventSynchronize(L->ev_pager));
    const int status = ((volatile int32_t *)L->h_mb)[0];
    if (status == WISP_ERR_OVERFLOW)
        return fail(WISP_ERR_OVERFLOW,
                    "wisp: per-kernel-call working set exceeds cap_experts (" +
                        std::to_string(L->cap) +
                        "); a single token routes to more unique experts than the cap, so the "
                        "forward cannot sub-batch it");
    if (status == WISP_ERR_BAD_EXPERT)
        return fail(WISP_ERR_BAD_EXPERT,
                    "wisp: routed expert id outside [0, " + std::to_string(L->E) + ")");
    if (status != WISP_OK) return fail(WISP_ERR_CUDA, "wisp: pager did not complete");
    return WISP_OK;
}

// Issue the page-ins of the mailbox's groups [g0, g1) and, when `compute` is
// set, the compute of each group.  `stream` is the caller's stream.
int page_and_compute(wisp_layer *L, const void *x, const float *w, int T, int K, void *out,
                     cudaStream_t stream, bool compute) {
    const int32_t *mb = L->h_mb;
    const int G = mb[1], nmiss = mb[2];
    const int32_t *grp = mb + kMbHeader;
    const int32_t *nu = grp + (T + 1);
    const int32_t *rec = mb + mailbox_miss_offset(T);
    int rc = ensure_events(L, std::max(G, 1));
    if (rc) return rc;
    int mi = 0;
    int64_t utot = 0;
    for (int g = 0; g < G; ++g) {
        const int t0 = grp[g], t1 = grp[g + 1];
        int wait_g = -1, m0 = mi;
        while (mi < nmiss && rec[4 * mi + 2] == g) {
            wait_g = std::max(wait_g, (int)rec[4 * mi + 3]);
            ++mi;
        }
        if (mi > m0) {
            if (wait_g >= 0) WISP_CUDA_TRY(cudaStreamWaitEvent(L->copy_stream, L->ev_group[wait_g], 0));
            for (int m = m0; m < mi; ++m) {
                const int64_t e = rec[4 * m], s = rec[4 * m + 1];
                WISP_CUDA_TRY(cudaMemcpyAsync(L->d13 + s * L->b13, L->h13 + e * L->b13, L->b13,
                                              cudaMemcpyHostToDevice, L->copy_stream));
                WISP_CUDA_TRY(cudaMemcpyAsync(L->d2 + s * L->b2, L->h2 + e * L->b2, L->b2,
                                              cudaMemcpyHostToDevice, L->copy_stream));
            }
            WISP_CUDA_TRY(cudaEventRecord(L->ev_copy[g], L->copy_stream));
            WISP_CUDA_TRY(cudaStreamWaitEvent(stream, L->ev_copy[g], 0));
        }
        utot += nu[g];
        if (compute && t1 > t0 && nu[g] > 0) {
            const int64_t p0 = (int64_t)t0 * K;
            GroupCompute gc{};
            gc.x = reinterpret_cast<const __nv_bfloat16 *>(x);
            gc.w13 = reinterpret_cast<const __nv_bfloat16 *>(L->d13);
            gc.w2 = reinterpret_cast<const __nv_bfloat16 *>(L->d2);
            gc.u_slot = L->d_u_slot + p0;
            gc.u_off = L->d_u_off + p0 + g;
            gc.u_pairs = L->d_u_pairs + p0;
            gc.nu = L->d_grp_nu + g;
            gc.topk_w = w;
            gc.act = L->d_act;
            gc.y = L->d_y;
            gc.out = reinterpret_cast<__nv_bfloat16 *>(out);
            gc.counters = L->d_counters;
            gc.K = K;
            gc.H = L->H;
            gc.I = L->I;
            gc.t0 = t0;
            gc.t1 = t1;
            rc = launch_decode_group(gc, nu[g], stream);
            if (rc) return rc;
        }
        WISP_CUDA_TRY(cudaEventRecord(L->ev_group[g], stream));
    }
    WISP_CUDA_TRY(cudaEventRecord(L->ev_copies, L->copy_stream));
    L->info[0] = G;
    L->info[1] = nmiss;
    L->info[2] = (int64_t)nmiss * (L->b13 + L->b2);
    L->info[3] = utot;
    return WISP_OK;
}

}  // namespace

extern "C" {

const char *wisp_version(void) { return "wisp_b200 0.1.0 (sm_100a)"; }

const char *wisp_last_error(void) { return g_last_error.c_str(); }

int wisp_layer_create(int32_t num_experts, int32_t cap_experts, int32_t hidden, int32_t inter,
                      int64_t w13_expert_bytes, int64_t w2_expert_bytes, const void *host_w13,
                      const void *host_w2, int32_t device, int32_t mode, wisp_layer **out) {
    if (!out) return fail(WISP_ERR_INVALID, "wisp_layer_create: out is NULL");
    *out = nullptr;
    if (num_experts < 1 || num_experts > 1024)
        return fail(WISP_ERR_INVALID, "wisp_layer_create: num_experts must be in [1, 1024]");
    if (cap_experts < 1 || cap_experts > num_experts)
        return fail(WISP_ERR_INVALID, "wisp_layer_create: cap_experts must be in [1, num_experts]");
    if (mode == WISP_MODE_RESIDENT && cap_experts != num_experts)
        return fail(WISP_ERR_INVALID, "wisp_layer_create: resident mode needs cap == num_experts");
    if (mode != WISP_MODE_PAGED && mode != WISP_MODE_RESIDENT)
        return fail(WISP_ERR_INVALID, "wisp_layer_create: unknown mode");
    if (w13_expert_bytes <= 0 || w2_expert_bytes <= 0 || !host_w13 || !host_w2)
        return fail(WISP_ERR_INVALID, "wisp_layer_create: empty expert weights");
    if (hidden < 0 || inter < 0)
        return fail(WISP_ERR_INVALID, "wisp_layer_create: negative shape");
    if (hidden > 0 && inter > 0) {
        if (hidden % 8 || inter % 8)
            return fail(WISP_ERR_UNSUPPORTED, "wisp_layer_create: hidden and inter must be multiples of 8");
        if (w13_expert_bytes != 2LL * 2 * inter * hidden || w2_expert_bytes != 2LL * hidden * inter)
            return fail(WISP_ERR_INVALID,
                        "wisp_layer_create: expert bytes do not match bf16 [2I,H] / [H,I]");
    }
    DeviceGuard guard(device);
    cudaPointerAttributes pa{};
    for (const void *hp : {host_w13, host_w2}) {
        if (cudaPointerGetAttributes(&pa, hp) != cudaSuccess || pa.type != cudaMemoryTypeHost) {
            cudaGetLastError();
            return fail(WISP_ERR_INVALID, "wisp_layer_create: host expert weights must be pinned");
        }
    }
    wisp_layer *L = new wisp_layer();
    L->dev = device;
    L->E = num_experts;
    L->cap = cap_experts;
    L->H = hidden;
    L->I = inter;
    L->mode = mode;
    L->b13 = w13_expert_bytes;
    L->b2 = w2_expert_bytes;
    L->h13 = reinterpret_cast<const char *>(host_w13);
    L->h2 = reinterpret_cast<const char *>(host_w2);
    auto bail = [&](int rc) {
        wisp_layer_destroy(L);
        return rc;
    };
    int rc = alloc_state(L, cap_experts);
    if (rc) return bail(rc == WISP_ERR_CUDA ? WISP_ERR_NOMEM : rc);
    if (cudaMalloc(&L->d_emap, sizeof(int32_t) * num_experts) != cudaSuccess ||
        cudaMalloc(&L->d_hdr, sizeof(int64_t) * 8) != cudaSuccess)
        return bail(fail(WISP_ERR_NOMEM, "wisp_layer_create: device allocation failed"));
    if (cudaMemset(L->d_emap, 0xff, sizeof(int32_t) * num_experts) != cudaSuccess ||
        cudaMemset(L->d_hdr, 0, sizeof(int64_t) * 8) != cudaSuccess ||
        cudaStreamCreateWithFlags(&L->copy_stream, cudaStreamNonBlocking) != cudaSuccess ||
        cudaEventCreateWithFlags(&L->ev_pager, cudaEventDisableTiming) !=
            cudaSuccess ||
        cudaEventCreateWithFlags(&L->ev_copies, cudaEventDisableTiming) != cudaSuccess)
        return bail(fail(WISP_ERR_CUDA, "wisp_layer_create: stream/event setup failed"));
    rc = ensure_ws(L, 16, 8);
    if (rc) return bail(rc);
    if (cudaDeviceSynchronize() != cudaSuccess)
        return bail(fail(WISP_ERR_CUDA, "wisp_layer_create: device sync failed"));
    *out = L;
    return WISP_OK;
}

int wisp_layer_destroy(wisp_layer *L) {
    if (!L) return WISP_OK;
    DeviceGuard guard(L->dev);
    cudaDeviceSynchronize();
    free_ws(L);
    cudaFree(L->d13);
    cudaFree(L->d2);
    cudaFree(L->d_s2e);
    cudaFree(L->d_tick);
    cudaFree(L->d_emap);
    cudaFree(L->d_hdr);
    for (auto e : L->ev_group) cudaEventDestroy(e);
    for (auto e : L->ev_copy) cudaEventDestroy(e);
    if (L->ev_pager) cudaEventDestroy(L->ev_pager);
    if (L->ev_copies) cudaEventDestroy(L->ev_copies);
    if (L->copy_stream) cudaStreamDestroy(L->copy_stream);
    delete L;
    return WISP_OK;
}

int wisp_moe_forward(wisp_layer *L, const void *x, const float *topk_weights,
                     const void *topk_ids, int32_t ids_int64, int32_t num_tokens, int32_t top_k,
                     void *out, void *stream) {
    if (!L) return fail(WISP_ERR_INVALID, "wisp_moe_forward: NULL layer");
    if (L->H <= 0 || L->I <= 0)
        return fail(WISP_ERR_UNSUPPORTED, "wisp_moe_forward: layer was created without a compute shape");
    if (num_tokens < 0 || top_k < 1 || top_k > 64)
        return fail(WISP_ERR_INVALID, "wisp_moe_forward: bad num_tokens/top_k");
    if (num_tokens > 0 && (!x || !topk_weights || !topk_ids || !out))
        return fail(WISP_ERR_INVALID, "wisp_moe_forward: NULL tensor");
    if (!aligned16(x) || !aligned16(out))
        return fail(WISP_ERR_INVALID, "wisp_moe_forward: x and out must be 16-byte aligned");
    std::lock_guard<std::mutex> lk(L->mu);
    DeviceGuard guard(L->dev);
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    int rc = run_pager(L, topk_ids, ids_int64, num_tokens, top_k, 0, 1, s);
    if (rc) return rc;
    return page_and_compute(L, x, topk_weights, num_tokens, top_k, out, s, true);
}

int wisp_ensure_resident(wisp_layer *L, const void *ids, int32_t ids_int64, int32_t n,
                         void *stream) {
    if (!L) return fail(WISP_ERR_INVALID, "wisp_ensure_resident: NULL layer");
    if (n < 0 || (n > 0 && !ids)) return fail(WISP_ERR_INVALID, "wisp_ensure_resident: bad ids");
    if (L->mode != WISP_MODE_PAGED)
        return fail(WISP_ERR_INVALID, "wisp_ensure_resident: layer is not in paged mode");
    std::lock_guard<std::mutex> lk(L->mu);
    DeviceGuard guard(L->dev);
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    int rc = run_pager(L, ids, ids_int64, 1, n, 1, 0, s);
    if (rc) return rc;
    rc = page_and_compute(L, nullptr, nullptr, 1, n, nullptr, s, false);
    if (rc) return rc;
    WISP_CUDA_TRY(cudaStreamSynchronize(L->copy_stream));
    WISP_CUDA_TRY(cudaStreamSynchronize(s));
    return WISP_OK;
}

int wisp_pager_step(wisp_layer *L, const void *topk_ids, int32_t ids_int64, int32_t num_tokens,
                    int32_t top_k, int32_t *slots_out, void *stream) {
    if (!L) return fail(WISP_ERR_INVALID, "wisp_pager_step: NULL layer");
    if (num_tokens < 0 || top_k < 1 || (num_tokens > 0 && !topk_ids))
        return fail(WISP_ERR_INVALID, "wisp_pager_step: bad ids");
    std::lock_guard<std::mutex> lk(L->mu);
    DeviceGuard guard(L->dev);
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    int rc = run_pager(L, topk_ids, ids_int64, num_tokens, top_k, 0, 1, s);
    if (rc) return rc;
    rc = page_and_compute(L, nullptr, nullptr, num_tokens, top_k, nullptr, s, false);
    if (rc) return rc;
    WISP_CUDA_TRY(cudaStreamSynchronize(L->copy_stream));
    WISP_CUDA_TRY(cudaStreamSynchronize(s));
    if (slots_out && num_tokens > 0)
        WISP_CUDA_TRY(cudaMemcpy(slots_out, L->d_slots, sizeof(int32_t) * (size_t)num_tokens * top_k,
                                 cudaMemcpyDeviceToHost));
    return WISP_OK;
}

int wisp_prime_identity(wisp_layer *L, void *stream) {
    if (!L) return fail(WISP_ERR_INVALID, "wisp_prime_identity: NULL layer");
    if (L->cap != L->E) return fail(WISP_ERR_INVALID, "prime_identity requires cap == num_experts");
    std::lock_guard<std::mutex> lk(L->mu);
    DeviceGuard guard(L->dev);
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    WISP_CUDA_TRY(cudaStreamWaitEvent(L->copy_stream, L->ev_copies, 0));
    WISP_CUDA_TRY(cudaMemcpyAsync(L->d13, L->h13, (size_t)L->E * L->b13, cudaMemcpyHostToDevice,
                                  L->copy_stream));
    WISP_CUDA_TRY(cudaMemcpyAsync(L->d2, L->h2, (size_t)L->E * L->b2, cudaMemcpyHostToDevice,
                                  L->copy_stream));
    fill_identity_kernel<<<(L->E + 255) / 256, 256, 0, L->copy_stream>>>(L->d_s2e, L->d_emap, L->E);
    WISP_CUDA_TRY(cudaGetLastError());
    WISP_CUDA_TRY(cudaEventRecord(L->ev_copies, L->copy_stream));
    WISP_CUDA_TRY(cudaStreamWaitEvent(s, L->ev_copies, 0));
    return WISP_OK;
}

int wisp_resize_cap(wisp_layer *L, int32_t new_cap, void *stream) {
    if (!L) return fail(WISP_ERR_INVALID, "wisp_resize_cap: NULL layer");
    (void)stream;
    std::lock_guard<std::mutex> lk(L->mu);
    DeviceGuard guard(L->dev);
    new_cap = std::max(2, std::min((int)new_cap, L->E));
    if (new_cap == L->cap) return WISP_OK;
    WISP_CUDA_TRY(cudaDeviceSynchronize());  // drained barrier, as the reference requires
    const int old = L->cap, keep = std::min(old, new_cap);
    std::vector<int32_t> s2e(old), emap(L->E);
    std::vector<int64_t> tick(old);
    WISP_CUDA_TRY(cudaMemcpy(s2e.data(), L->d_s2e, sizeof(int32_t) * old, cudaMemcpyDeviceToHost));
    WISP_CUDA_TRY(cudaMemcpy(tick.data(), L->d_tick, sizeof(int64_t) * old, cudaMemcpyDeviceToHost));
    WISP_CUDA_TRY(cudaMemcpy(emap.data(), L->d_emap, sizeof(int32_t) * L->E, cudaMemcpyDeviceToHost));
    char *o13 = L->d13, *o2 = L->d2;
    int32_t *os2e = L->d_s2e;
    int64_t *otick = L->d_tick;
    L->d13 = L->d2 = nullptr;
    int rc = alloc_state(L, new_cap);
    if (rc) {
        cudaFree(L->d13);
        cudaFree(L->d2);
        cudaFree(L->d_s2e);
        cudaFree(L->d_tick);
        L->d13 = o13;
        L->d2 = o2;
        L->d_s2e = os2e;
        L->d_tick = otick;
        return WISP_ERR_NOMEM;
    }
    WISP_CUDA_TRY(cudaMemcpy(L->d13, o13, (size_t)keep * L->b13, cudaMemcpyDeviceToDevice));
    WISP_CUDA_TRY(cudaMemcpy(L->d2, o2, (size_t)keep * L->b2, cudaMemcpyDeviceToDevice));
    if (new_cap < old) {
        for (int s = new_cap; s < old; ++s)
            if (s2e[s] >= 0) emap[s2e[s]] = -1;
    }
    s2e.resize(new_cap, -1);
    tick.resize(new_cap, 0);
    WISP_CUDA_TRY(cudaMemcpy(L->d_s2e, s2e.data(), sizeof(int32_t) * new_cap, cudaMemcpyHostToDevice));
    WISP_CUDA_TRY(cudaMemcpy(L->d_tick, tick.data(), sizeof(int64_t) * new_cap, cudaMemcpyHostToDevice));
    WISP_CUDA_TRY(cudaMemcpy(L->d_emap, emap.data(), sizeof(int32_t) * L->E, cudaMemcpyHostToDevice));
    cudaFree(o13);
    cudaFree(o2);
    cudaFree(os2e);
    cudaFree(otick);
    L->cap = new_cap;
    return WISP_OK;
}

int wisp_get_state(wisp_layer *L, int32_t *slot_to_expert, int64_t *lru_tick, int64_t *clock,
                   int64_t *stats4, int32_t *expert_map, int32_t *cap) {
    if (!L) return fail(WISP_ERR_INVALID, "wisp_get_state: NULL layer");
    std::lock_guard<std::mutex> lk(L->mu);
    DeviceGuard guard(L->dev);
    WISP_CUDA_TRY(cudaDeviceSynchronize());
    if (cap) *cap = L->cap;
    if (slot_to_expert)
        WISP_CUDA_TRY(cudaMemcpy(slot_to_expert, L->d_s2e, sizeof(int32_t) * L->cap, cudaMemcpyDeviceToHost));
    if (lru_tick)
        WISP_CUDA_TRY(cudaMemcpy(lru_tick, L->d_tick, sizeof(int64_t) * L->cap, cudaMemcpyDeviceToHost));
    if (expert_map)
        WISP_CUDA_TRY(cudaMemcpy(expert_map, L->d_emap, sizeof(int32_t) * L->E, cudaMemcpyDeviceToHost));
    int64_t hdr[5];
    WISP_CUDA_TRY(cudaMemcpy(hdr, L->d_hdr, sizeof(hdr), cudaMemcpyDeviceToHost));
    if (clock) *clock = hdr[0];
    if (stats4)
        for (int i = 0; i < 4; ++i) stats4[i] = hdr[1 + i];
    return WISP_OK;
}

int wisp_set_stats(wisp_layer *L, const int64_t *stats4) {
    if (!L || !stats4) return fail(WISP_ERR_INVALID, "wisp_set_stats: NULL argument");
    std::lock_guard<std::mutex> lk(L->mu);
    DeviceGuard guard(L->dev);
    WISP_CUDA_TRY(cudaDeviceSynchronize());
    WISP_CUDA_TRY(cudaMemcpy(L->d_hdr + 1, stats4, sizeof(int64_t) * 4, cudaMemcpyHostToDevice));
    return WISP_OK;
}

int wisp_layer_buffers(wisp_layer *L, void **scratch_w13, void **scratch_w2, void **expert_map) {
    if (!L) return fail(WISP_ERR_INVALID, "wisp_layer_buffers: NULL layer");
    if (scratch_w13) *scratch_w13 = L->d13;
    if (scratch_w2) *scratch_w2 = L->d2;
    if (expert_map) *expert_map = L->d_emap;
    return WISP_OK;
}

int wisp_last_forward_info(wisp_layer *L, int64_t *info4) {
    if (!L || !info4) return fail(WISP_ERR_INVALID, "wisp_last_forward_info: NULL argument");
    for (int i = 0; i < 4; ++i) info4[i] = L->info[i];
    return WISP_OK;
}

}  // extern "C"
