// dp_peer.cu -- data-parallel optimiser step over peer memory (NVLink).
//
// Every rank (one process per GPU) holds a replica of the Gaussians and has
// just written its view's gradient buffer (msplat_train_step_grads).  Instead
// of an all-reduce of the whole buffer followed by Adam on every replica,
// each rank owns 1/world of the Gaussians and, in one kernel, reads the
// world gradient shards of its Gaussians straight from the peers' memory,
// sums them, runs Adam with its own moments, and stores the updated
// parameters into every replica (its own and the peers').  Per GPU that moves
// about 2 x (world-1)/world of one buffer over NVLink and does 1/world of the
// Adam work.
//
// Ordering between GPUs uses one flag array per rank in its own memory,
// written by the peers with system-scope atomics and polled locally:
//   phase 0  "my gradients are complete"   (signal kernel after the gradients)
//   phase 1  "my shard is in every replica" (last CTA of the update kernel)
// A rank's next step may only start once it has seen every phase-1 flag:
// then every peer has finished reading its gradient buffer and writing into
// its parameters.  Each flag holds the step number (epoch), so flags never
// need resetting.  Every wait is bounded by the GPU's global timer; a wait
// that runs out sets a bit in this file's error word and the kernel returns,
// which leaves the GPU usable and the step's update incomplete.
//
// Buffers shared this way must be whole allocations (msplat_gpu_alloc);
// their IPC handles are exchanged by the host (torch.distributed).
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdio>
#include <cstring>
#include <map>
#include <string>

#include "../../include/msplat_engine.h"
#include "adam.cuh"
#include "engine.h"
#include "msp_math.cuh"

namespace msp {
namespace {

constexpr int kMaxRanks = 8;
constexpr int kDpThreads = 256;

enum DpError : int {
    kDpWaitGrads = 1,   // a peer's gradients did not arrive in time
    kDpWaitShards = 2,  // a peer's updated shard did not arrive in time
};

struct DpArgs {
    const float* grads[kMaxRanks];           // every rank's gradient buffer
    float* params[kMaxRanks][kGroups];       // every rank's parameter arrays
    float* exp_avg[kGroups];                 // this rank's moments
    float* exp_avg_sq[kGroups];
    unsigned* flags[kMaxRanks];              // every rank's flag array [2 * world]
    float step[kGroups], inv_bc2[kGroups];
    int stride[kGroups];
    long long goff[kGroups];                 // group offsets in the gradient buffer
    long long vis_off;                       // visibility flags' offset
    long long cam_off;                       // compact form: camera position's offset
    int rest_stride;                         // floats per Gaussian of features_rest
    int rank, world, begin, end, used_rest;
    int vec;                                 // bit g: group g's arrays are 16-byte aligned
    float b1, b2, eps, scale;
    unsigned epoch;
    unsigned long long timeout_ns;
    int* err;                                // this rank's DP error word
    unsigned* done_ctas;                     // this rank's CTA counter
};

__device__ __forceinline__ unsigned long long global_ns()
{
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ unsigned load_acquire_sys(const unsigned* p)
{
    unsigned v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// Waits until every rank's entry of `phase` in this rank's flag array has
// reached the epoch; false if the global timer passes the limit first.
__device__ bool wait_all(const DpArgs& a, int phase)
{
    const unsigned* f = a.flags[a.rank] + phase * a.world;
    const unsigned long long t0 = global_ns();
    for (int q = 0; q < a.world; q++) {
        while (load_acquire_sys(f + q) < a.epoch) {
            if (global_ns() - t0 > a.timeout_ns) return false;
            __nanosleep(128);
        }
    }
    return true;
}

// Publishes this rank's `phase` entry (the epoch) in every rank's flag array.
__device__ void signal_all(const DpArgs& a, int phase)
{
    __threadfence_system();
    for (int q = 0; q < a.world; q++) atomicMax_system(a.flags[q] + phase * a.world + a.rank, a.epoch);
}

__global__ void dp_signal_kernel(DpArgs a, int phase)
{
    if (threadIdx.x == 0) signal_all(a, phase);
}

__global__ void dp_wait_kernel(DpArgs a, int phase, int errbit)
{
    if (threadIdx.x == 0 && !wait_all(a, phase)) atomicOr(a.err, errbit);
}

// Sum of the ranks' gradients for element e of a group, rank order 0..world-1
// (the same on every rank: each element has one owner).
__device__ __forceinline__ float rank_sum(const DpArgs& a, long long off)
{
    float g = a.grads[0][off];
    for (int q = 1; q < a.world; q++) g += a.grads[q][off];
    return g;
}

__device__ __forceinline__ float4 ld4(const float* p) { return *reinterpret_cast<const float4*>(p); }
__device__ __forceinline__ void st4(float* p, float4 v) { *reinterpret_cast<float4*>(p) = v; }
__device__ __forceinline__ float& comp(float4& v, int k)
{
    return k == 0 ? v.x : k == 1 ? v.y : k == 2 ? v.z : v.w;
}

// Phase-0 wait, then the shard's visibility: vis[i - begin] = 1 when some
// rank saw Gaussian i (its flags summed over the ranks, rank order).
__global__ void __launch_bounds__(kDpThreads)
dp_vis_kernel(DpArgs a, unsigned char* __restrict__ vis)
{
    __shared__ int s_ok;
    if (threadIdx.x == 0) {
        s_ok = wait_all(a, 0);
        if (!s_ok) atomicOr(a.err, kDpWaitGrads);
    }
    __syncthreads();
    if (!s_ok) return;
    for (int i = a.begin + blockIdx.x * blockDim.x + threadIdx.x; i < a.end;
         i += gridDim.x * blockDim.x)
        vis[i - a.begin] = rank_sum(a, a.vis_off + i) > 0.f ? 1 : 0;
}

// Whether element e of group gi (shard-relative element index rel) is
// updated: SH groups only for Gaussians some rank saw, features_rest only for
// the SH degrees in use.
__device__ __forceinline__ bool updated(const DpArgs& a, int gi, int S,
                                        const unsigned char* __restrict__ vis, long long rel)
{
    if (gi != 3 && gi != 4) return true;
    const long long il = rel / S;
    return vis[il] && (gi != 4 || rel - il * S < a.used_rest);
}

template <int W>
__device__ __forceinline__ void update_scalar(const DpArgs& a, int gi, int S,
                                              const unsigned char* __restrict__ vis,
                                              long long e0s, long long rel)
{
    if (!updated(a, gi, S, vis, rel)) return;
    const long long e = e0s + rel;
    float p = a.params[a.rank][gi][e], m = a.exp_avg[gi][e], v = a.exp_avg_sq[gi][e];
    float g = a.grads[0][a.goff[gi] + e];
#pragma unroll
    for (int q = 1; q < W; q++) g += a.grads[q][a.goff[gi] + e];
    adam_math(p, m, v, g * a.scale, a.step[gi], a.b1, a.b2, a.inv_bc2[gi], a.eps);
    a.exp_avg[gi][e] = m;
    a.exp_avg_sq[gi][e] = v;
#pragma unroll
    for (int q = 0; q < W; q++) a.params[q][gi][e] = p;
}

// Elements [rel, rel+4) of the shard's slice of group gi with 16-byte loads
// and stores; every rank's gradient vector (most of them remote) is
// requested before any is used.  Elements that are not updated are stored
// back unchanged.
template <int W>
__device__ __forceinline__ void update_vec4(const DpArgs& a, int gi, int S,
                                            const unsigned char* __restrict__ vis, long long e0s,
                                            long long rel)
{
    const long long e0 = e0s + rel;
    float4 gq[W];
#pragma unroll
    for (int q = 0; q < W; q++) gq[q] = ld4(a.grads[q] + a.goff[gi] + e0);
    float4 p = ld4(a.params[a.rank][gi] + e0);
    float4 m = ld4(a.exp_avg[gi] + e0), v = ld4(a.exp_avg_sq[gi] + e0);
    float4 g = gq[0];
#pragma unroll
    for (int q = 1; q < W; q++) {
        g.x += gq[q].x;
        g.y += gq[q].y;
        g.z += gq[q].z;
        g.w += gq[q].w;
    }
#pragma unroll
    for (int k = 0; k < 4; k++)
        if (updated(a, gi, S, vis, rel + k))
            adam_math(comp(p, k), comp(m, k), comp(v, k), comp(g, k) * a.scale, a.step[gi], a.b1,
                      a.b2, a.inv_bc2[gi], a.eps);
    st4(a.exp_avg[gi] + e0, m);
    st4(a.exp_avg_sq[gi] + e0, v);
#pragma unroll
    for (int q = 0; q < W; q++) st4(a.params[q][gi] + e0, p);
}

// kDpU vector elements per thread per round (elements v, v + nthreads, ...):
// every load of the round -- each rank's gradient vector, most of them
// remote, and the local parameter and moments -- is issued before any
// store, so a thread keeps kDpU * world remote loads in flight.  (Two
// update_vec4 calls in a row do not: the compiler cannot move the second's
// loads above the first's stores into the replicas, which may alias.)
constexpr int kDpU = 2;
template <int W, int U>
__device__ __forceinline__ void update_vec4_batch(const DpArgs& a, int gi, int S,
                                                  const unsigned char* __restrict__ vis,
                                                  long long e0s, long long v0, long long stride,
                                                  long long nvec)
{
    float4 g[U], p[U], m[U], vv[U];
#pragma unroll
    for (int u = 0; u < U; u++) {
        const long long vi = v0 + u * stride;
        if (vi >= nvec) continue;
        const long long e0 = e0s + 4 * vi;
        float4 gq[W];
#pragma unroll
        for (int q = 0; q < W; q++) gq[q] = ld4(a.grads[q] + a.goff[gi] + e0);
        p[u] = ld4(a.params[a.rank][gi] + e0);
        m[u] = ld4(a.exp_avg[gi] + e0);
        vv[u] = ld4(a.exp_avg_sq[gi] + e0);
        g[u] = gq[0];
#pragma unroll
        for (int q = 1; q < W; q++) {
            g[u].x += gq[q].x;
            g[u].y += gq[q].y;
            g[u].z += gq[q].z;
            g[u].w += gq[q].w;
        }
    }
#pragma unroll
    for (int u = 0; u < U; u++) {
        const long long vi = v0 + u * stride;
        if (vi >= nvec) continue;
        const long long rel = 4 * vi;
        const long long e0 = e0s + rel;
#pragma unroll
        for (int k = 0; k < 4; k++)
            if (updated(a, gi, S, vis, rel + k))
                adam_math(comp(p[u], k), comp(m[u], k), comp(vv[u], k), comp(g[u], k) * a.scale,
                          a.step[gi], a.b1, a.b2, a.inv_bc2[gi], a.eps);
        st4(a.exp_avg[gi] + e0, m[u]);
        st4(a.exp_avg_sq[gi] + e0, vv[u]);
#pragma unroll
        for (int q = 0; q < W; q++) st4(a.params[q][gi] + e0, p[u]);
    }
}

// The update of the shard, group by group, as one flat vector stream per
// group (no barriers); skipped when the phase-0 wait failed.
template <int W>
__global__ void __launch_bounds__(kDpThreads, 3)
dp_reduce_adam_kernel(DpArgs a, const unsigned char* __restrict__ vis)
{
    const bool ok = (*(volatile int*)a.err & kDpWaitGrads) == 0;
    if (ok) {
        const long long tid = (long long)blockIdx.x * blockDim.x + threadIdx.x;
        const long long nthreads = (long long)gridDim.x * blockDim.x;
        for (int gi = 0; gi < kGroups; gi++) {
            if (!a.params[a.rank][gi]) continue;
            const int S = a.stride[gi];
            const long long e0s = (long long)a.begin * S;  // a multiple of 4: begin is of 32
            const long long total = (long long)(a.end - a.begin) * S;
            long long body = 0;
            if (a.vec & (1 << gi)) {
                body = total / 4 * 4;
                const long long nvec = body / 4;
                for (long long v = tid; v < nvec; v += kDpU * nthreads)
                    update_vec4_batch<W, kDpU>(a, gi, S, vis, e0s, v, nthreads, nvec);
            }
            for (long long rel = body + tid; rel < total; rel += nthreads)
                update_scalar<W>(a, gi, S, vis, e0s, rel);
        }
    }
    // the last CTA to finish publishes phase 1 for this rank
    __threadfence_system();
    __syncthreads();
    if (threadIdx.x == 0) {
        const unsigned prev = atomicAdd(a.done_ctas, 1u);
        if (prev == gridDim.x - 1) {
            *a.done_ctas = 0;
            if (ok) signal_all(a, 1);
        }
    }
}

// Compact form.  Each rank's buffer holds, per Gaussian, the gradients of
// means, scales, quats and opacity, v_rgb (the colour gradient) and a
// visibility flag, plus the rank's camera position.  The gradient of every
// SH coefficient of a view is v_rgb times a basis value of that view's
// direction to the mean, so the owner of a Gaussian rebuilds each rank's
// dc and features_rest gradients (C0 * v_rgb, basis[b] * v_rgb[c]) from its
// pre-update mean and sums them in rank order, exactly as the full buffer
// would have carried them -- while 4x fewer bytes cross NVLink.
constexpr int kCompactG = 256;   // Gaussians per work chunk (one per thread)

template <int W>
__global__ void __launch_bounds__(kDpThreads, 2)
dp_compact_kernel(DpArgs a)
{
    extern __shared__ float s_rest[];               // [kCompactG][rsp] rest gradients
    __shared__ float s_dc[kCompactG][3];
    __shared__ unsigned char s_vis[kCompactG];
    __shared__ float s_cam[W][3];
    const bool ok = (*(volatile int*)a.err & kDpWaitGrads) == 0;
    const int rs = a.rest_stride, rsp = rs | 1;
    if (ok) {
        const int tid = threadIdx.x;
        if (tid < 3 * W) s_cam[tid / 3][tid % 3] = a.grads[tid / 3][a.cam_off + tid % 3];
        const int nchunks = (a.end - a.begin + kCompactG - 1) / kCompactG;
        for (int ch = blockIdx.x; ch < nchunks; ch += gridDim.x) {
            const int c0 = a.begin + ch * kCompactG;
            const int cn = min(kCompactG, a.end - c0);
            __syncthreads();
            // phase A: this thread's Gaussian
            if (tid < cn) {
                const long long i = c0 + tid;
                float vsum = a.grads[0][a.vis_off + i];
#pragma unroll
                for (int q = 1; q < W; q++) vsum += a.grads[q][a.vis_off + i];
                const bool vis = vsum > 0.f;
                s_vis[tid] = vis;
                if (vis) {
                    const float* mp = a.params[a.rank][0] + 3 * i;
                    const float p[3] = {mp[0], mp[1], mp[2]};
                    float* row = s_rest + tid * rsp;
#pragma unroll 1
                    for (int q = 0; q < W; q++) {
                        const float* vr = a.grads[q] + a.goff[3] + 3 * i;
                        const float v0 = vr[0], v1 = vr[1], v2 = vr[2];
                        const float d0 = MSP_SH_C0 * v0, d1 = MSP_SH_C0 * v1, d2 = MSP_SH_C0 * v2;
                        if (q == 0) {
                            s_dc[tid][0] = d0;
                            s_dc[tid][1] = d1;
                            s_dc[tid][2] = d2;
                        } else {
                            s_dc[tid][0] += d0;
                            s_dc[tid][1] += d1;
                            s_dc[tid][2] += d2;
                        }
                        if (a.used_rest > 0) {
                            float bs[15];
                            sh_rest_basis(s_cam[q], p, bs);
                            for (int kk = 0; kk < a.used_rest; kk++) {
                                const int b = kk / 3, c = kk - 3 * b;
                                const float g = bs[b] * (c == 0 ? v0 : c == 1 ? v1 : v2);
                                row[kk] = q == 0 ? g : row[kk] + g;
                            }
                        }
                    }
                }
            }
            __syncthreads();
            // phase B: the chunk's slice of every group
            for (int gi = 0; gi < kGroups; gi++) {
                if (!a.params[a.rank][gi]) continue;
                const int S = a.stride[gi];
                const long long e0s = (long long)c0 * S;
                const int total = cn * S;
                if (gi == 3 || gi == 4) {
                    // gradients from shared memory; 16-byte parameter and
                    // moment traffic, two vectors per thread per round
                    auto sh_grad = [&](int rel, float& g) {
                        const int il = rel / S, kk = rel - il * S;
                        if (!s_vis[il] || (gi == 4 && kk >= a.used_rest)) return false;
                        g = gi == 3 ? s_dc[il][kk] : s_rest[il * rsp + kk];
                        return true;
                    };
                    int body = 0;
                    if (a.vec & (1 << gi)) {
                        body = total / 4 * 4;
                        const int nvec = body / 4;
                        for (int v0 = tid; v0 < nvec; v0 += 2 * kDpThreads) {
                            float4 pv[2], mv[2], vv[2];
                            bool on[2];
#pragma unroll
                            for (int u = 0; u < 2; u++) {
                                const int vi = v0 + u * kDpThreads;
                                on[u] = vi < nvec;
                                if (!on[u]) continue;
                                const long long e = e0s + 4 * vi;
                                pv[u] = ld4(a.params[a.rank][gi] + e);
                                mv[u] = ld4(a.exp_avg[gi] + e);
                                vv[u] = ld4(a.exp_avg_sq[gi] + e);
                            }
#pragma unroll
                            for (int u = 0; u < 2; u++) {
                                if (!on[u]) continue;
                                const int vi = v0 + u * kDpThreads;
#pragma unroll
                                for (int k = 0; k < 4; k++) {
                                    float g;
                                    if (sh_grad(4 * vi + k, g))
                                        adam_math(comp(pv[u], k), comp(mv[u], k), comp(vv[u], k),
                                                  g * a.scale, a.step[gi], a.b1, a.b2,
                                                  a.inv_bc2[gi], a.eps);
                                }
                                const long long e = e0s + 4 * vi;
                                st4(a.exp_avg[gi] + e, mv[u]);
                                st4(a.exp_avg_sq[gi] + e, vv[u]);
#pragma unroll
                                for (int q = 0; q < W; q++) st4(a.params[q][gi] + e, pv[u]);
                            }
                        }
                    }
                    for (int rel = body + tid; rel < total; rel += kDpThreads) {
                        float g;
                        if (!sh_grad(rel, g)) continue;
                        const long long e = e0s + rel;
                        float p = a.params[a.rank][gi][e], m = a.exp_avg[gi][e],
                              v = a.exp_avg_sq[gi][e];
                        adam_math(p, m, v, g * a.scale, a.step[gi], a.b1, a.b2, a.inv_bc2[gi],
                                  a.eps);
                        a.exp_avg[gi][e] = m;
                        a.exp_avg_sq[gi][e] = v;
#pragma unroll
                        for (int q = 0; q < W; q++) a.params[q][gi][e] = p;
                    }
                    continue;
                }
                // means, scales, quats, opacity: the ranks' gradients, summed here
                long long body = 0;
                if (a.vec & (1 << gi)) {
                    body = total / 4 * 4;
                    const int nvec = (int)(body / 4);
                    for (int v = tid; v < nvec; v += 2 * kDpThreads) {
                        update_vec4<W>(a, gi, S, nullptr, e0s, 4 * v);
                        if (v + kDpThreads < nvec) update_vec4<W>(a, gi, S, nullptr, e0s, 4 * (v + kDpThreads));
                    }
                }
                for (long long rel = body + tid; rel < total; rel += kDpThreads)
                    update_scalar<W>(a, gi, S, nullptr, e0s, rel);
            }
        }
    }
    // the last CTA to finish publishes phase 1 for this rank
    __threadfence_system();
    __syncthreads();
    if (threadIdx.x == 0) {
        const unsigned prev = atomicAdd(a.done_ctas, 1u);
        if (prev == gridDim.x - 1) {
            *a.done_ctas = 0;
            if (ok) signal_all(a, 1);
        }
    }
}

// Per-device DP state: the error word and the CTA counter.
struct DpState {
    int* err = nullptr;
    unsigned* done = nullptr;
    unsigned char* vis = nullptr;  // shard visibility
    long long vis_cap = 0;
};
DpState g_dp[kMaxRanks * 4];
std::map<std::string, void*> g_opened;  // IPC handle bytes -> mapped pointer

#define DP_CUDA(expr)                                                                     \
    do {                                                                                  \
        cudaError_t e_ = (expr);                                                          \
        if (e_ != cudaSuccess) {                                                          \
            set_error("%s failed: %s", #expr, cudaGetErrorString(e_));                    \
            return MSPLAT_ERR_CUDA;                                                       \
        }                                                                                 \
    } while (0)

int dp_state(DpState** st)
{
    int dev = 0;
    DP_CUDA(cudaGetDevice(&dev));
    if (dev < 0 || dev >= kMaxRanks * 4) {
        set_error("device %d out of range", dev);
        return MSPLAT_ERR_ARG;
    }
    DpState& s = g_dp[dev];
    if (!s.err) {
        DP_CUDA(cudaMalloc(&s.err, sizeof(int)));
        DP_CUDA(cudaMalloc(&s.done, sizeof(unsigned)));
        DP_CUDA(cudaMemset(s.err, 0, sizeof(int)));
        DP_CUDA(cudaMemset(s.done, 0, sizeof(unsigned)));
    }
    *st = &s;
    return MSPLAT_OK;
}

}  // namespace
}  // namespace msp

using namespace msp;

extern "C" {

int msplat_ipc_get_handle(const void* dev_ptr, void* handle_out)
{
    if (!dev_ptr || !handle_out) {
        set_error("msplat_ipc_get_handle: null pointer");
        return MSPLAT_ERR_ARG;
    }
    cudaIpcMemHandle_t h;
    DP_CUDA(cudaIpcGetMemHandle(&h, const_cast<void*>(dev_ptr)));
    memcpy(handle_out, &h, sizeof(h));
    return MSPLAT_OK;
}

int msplat_ipc_open_handle(const void* handle, void** dev_ptr_out)
{
    if (!handle || !dev_ptr_out) {
        set_error("msplat_ipc_open_handle: null pointer");
        return MSPLAT_ERR_ARG;
    }
    std::lock_guard<std::mutex> lk(engine_mutex());
    const std::string key(static_cast<const char*>(handle), sizeof(cudaIpcMemHandle_t));
    auto it = g_opened.find(key);
    if (it != g_opened.end()) {
        *dev_ptr_out = it->second;
        return MSPLAT_OK;
    }
    cudaIpcMemHandle_t h;
    memcpy(&h, handle, sizeof(h));
    void* p = nullptr;
    DP_CUDA(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess));
    g_opened[key] = p;
    *dev_ptr_out = p;
    return MSPLAT_OK;
}

int msplat_ipc_close_all(void)
{
    std::lock_guard<std::mutex> lk(engine_mutex());
    int rc = MSPLAT_OK;
    for (auto& kv : g_opened)
        if (cudaIpcCloseMemHandle(kv.second) != cudaSuccess) rc = MSPLAT_ERR_CUDA;
    g_opened.clear();
    if (rc) set_error("cudaIpcCloseMemHandle failed");
    return rc;
}

int msplat_dp_reduce_adam(int rank, int world, int num_points, int features_rest_bases,
                          unsigned degree, unsigned degrees_to_use,
                          const float* const* rank_grads, float* const* rank_params,
                          float* const* exp_avg, float* const* exp_avg_sq,
                          unsigned* const* rank_flags, unsigned epoch,
                          const float* step_sizes, const float* bc2_sqrts, float beta1,
                          float beta2, float eps, int compact, double timeout_s)
{
    std::lock_guard<std::mutex> lk(engine_mutex());
    int rc = engine_init();
    if (rc) return rc;
    const long long rs = (long long)features_rest_bases * 3;
    if (world < 1 || world > kMaxRanks || rank < 0 || rank >= world || num_points < 0 ||
        features_rest_bases < 0 || !rank_grads || !rank_params || !exp_avg || !exp_avg_sq ||
        !rank_flags || !step_sizes || !bc2_sqrts || epoch == 0 || !(timeout_s > 0.0)) {
        set_error("msplat_dp_reduce_adam: invalid arguments (rank %d of %d, N=%d, epoch %u)",
                  rank, world, num_points, epoch);
        return MSPLAT_ERR_ARG;
    }
    DpState* st = nullptr;
    if ((rc = dp_state(&st))) return rc;
    DpArgs a{};
    const int strides[kGroups] = {3, 3, 4, 3, (int)rs, 1};
    long long off = 0;
    for (int gi = 0; gi < kGroups; gi++) {
        a.stride[gi] = strides[gi];
        a.goff[gi] = off;
        off += (long long)strides[gi] * num_points;
        a.step[gi] = step_sizes[gi];
        a.inv_bc2[gi] = 1.0f / bc2_sqrts[gi];
        a.exp_avg[gi] = exp_avg[gi];
        a.exp_avg_sq[gi] = exp_avg_sq[gi];
    }
    a.vis_off = off;
    a.rest_stride = (int)rs;
    if (compact) {
        // means, scales, quats, v_rgb, opacities, visibility, camera
        const long long n = num_points;
        a.goff[0] = 0;
        a.goff[1] = 3 * n;
        a.goff[2] = 6 * n;
        a.goff[3] = 10 * n;
        a.goff[4] = 0;
        a.goff[5] = 13 * n;
        a.vis_off = 14 * n;
        a.cam_off = 15 * n;
    }
    for (int q = 0; q < world; q++) {
        a.grads[q] = rank_grads[q];
        a.flags[q] = rank_flags[q];
        if (!a.grads[q] || !a.flags[q]) {
            set_error("msplat_dp_reduce_adam: null pointer for rank %d", q);
            return MSPLAT_ERR_ARG;
        }
        for (int gi = 0; gi < kGroups; gi++) {
            a.params[q][gi] = strides[gi] ? rank_params[q * kGroups + gi] : nullptr;
            if (strides[gi] && !a.params[q][gi]) {
                set_error("msplat_dp_reduce_adam: null parameter array (rank %d, group %d)", q, gi);
                return MSPLAT_ERR_ARG;
            }
        }
    }
    for (int gi = 0; gi < kGroups; gi++)
        if (a.params[rank][gi] && (!a.exp_avg[gi] || !a.exp_avg_sq[gi])) {
            set_error("msplat_dp_reduce_adam: null moment array (group %d)", gi);
            return MSPLAT_ERR_ARG;
        }
    // shard: whole warps of Gaussians per rank
    const long long per = ((long long)num_points + world - 1) / world;
    const long long chunk = (per + 31) / 32 * 32;
    a.begin = (int)std::min<long long>((long long)rank * chunk, num_points);
    a.end = (int)std::min<long long>((long long)(rank + 1) * chunk, num_points);
    // 16-byte vectors for a group when every array it touches allows them
    for (int gi = 0; gi < kGroups; gi++) {
        if (!a.params[rank][gi]) continue;
        uintptr_t mis = (uintptr_t)a.exp_avg[gi] | (uintptr_t)a.exp_avg_sq[gi];
        for (int q = 0; q < world; q++) {
            mis |= (uintptr_t)a.params[q][gi];
            // compact form: the SH groups' gradients come from shared memory
            if (!(compact && (gi == 3 || gi == 4))) mis |= (uintptr_t)(a.grads[q] + a.goff[gi]);
        }
        if ((mis & 15) == 0) a.vec |= 1 << gi;
    }
    const int dtu = (int)std::min(degrees_to_use, degree);
    a.used_rest = rest_bases_updated(dtu, (int)rs) * 3;
    a.rank = rank;
    a.world = world;
    a.b1 = beta1;
    a.b2 = beta2;
    a.eps = eps;
    a.scale = 1.0f / (float)world;
    a.epoch = epoch;
    a.timeout_ns = (unsigned long long)(timeout_s * 1e9);
    a.err = st->err;
    a.done_ctas = st->done;
    const cudaStream_t s = engine_stream();
    dp_signal_kernel<<<1, 32, 0, s>>>(a, 0);
    if (compact) {
        const int rsp = (int)rs | 1;
        const size_t smem = (size_t)kCompactG * rsp * sizeof(float);
        const int nchunks = std::max(1, (a.end - a.begin + kCompactG - 1) / kCompactG);
        const int grid = std::min(nchunks, 148 * 2);
        dp_signal_kernel<<<1, 32, 0, s>>>(a, 0);
        dp_wait_kernel<<<1, 32, 0, s>>>(a, 0, kDpWaitGrads);
#define MSP_COMPACT(W)                                                                          \
    do {                                                                                        \
        static std::once_flag once_[kMaxDeviceSlots];                                           \
        static cudaError_t set_err_[kMaxDeviceSlots];                                           \
        int dev_ = 0;                                                                           \
        if (!once_per_device(once_, [](int d) {                                                 \
                set_err_[d] = cudaFuncSetAttribute(dp_compact_kernel<W>,                        \
                                                   cudaFuncAttributeMaxDynamicSharedMemorySize, \
                                                   96 * 1024);                                  \
            }))                                                                                 \
            DP_CUDA(cudaErrorNoDevice);                                                         \
        DP_CUDA(cudaGetDevice(&dev_));                                                          \
        DP_CUDA(set_err_[dev_]);                                                                \
        dp_compact_kernel<W><<<grid, kDpThreads, smem, s>>>(a);                                 \
    } while (0)
        switch (world) {
            case 1: MSP_COMPACT(1); break;
            case 2: MSP_COMPACT(2); break;
            case 3: MSP_COMPACT(3); break;
            case 4: MSP_COMPACT(4); break;
            case 5: MSP_COMPACT(5); break;
            case 6: MSP_COMPACT(6); break;
            case 7: MSP_COMPACT(7); break;
            default: MSP_COMPACT(8); break;
        }
#undef MSP_COMPACT
        dp_wait_kernel<<<1, 32, 0, s>>>(a, 1, kDpWaitShards);
        engine_add_launches(4);
        DP_CUDA(cudaGetLastError());
        return MSPLAT_OK;
    }
    const long long shard = a.end - a.begin;
    if (shard > st->vis_cap) {
        if (st->vis) cudaFree(st->vis);
        st->vis = nullptr;
        st->vis_cap = 0;
        DP_CUDA(cudaMalloc(&st->vis, (size_t)std::max(shard, 1LL)));
        st->vis_cap = shard;
    }
    dp_vis_kernel<<<148 * 2, kDpThreads, 0, s>>>(a, st->vis);
    const int grid = 148 * 3;
    switch (world) {
        case 1: dp_reduce_adam_kernel<1><<<grid, kDpThreads, 0, s>>>(a, st->vis); break;
        case 2: dp_reduce_adam_kernel<2><<<grid, kDpThreads, 0, s>>>(a, st->vis); break;
        case 3: dp_reduce_adam_kernel<3><<<grid, kDpThreads, 0, s>>>(a, st->vis); break;
        case 4: dp_reduce_adam_kernel<4><<<grid, kDpThreads, 0, s>>>(a, st->vis); break;
        case 5: dp_reduce_adam_kernel<5><<<grid, kDpThreads, 0, s>>>(a, st->vis); break;
        case 6: dp_reduce_adam_kernel<6><<<grid, kDpThreads, 0, s>>>(a, st->vis); break;
        case 7: dp_reduce_adam_kernel<7><<<grid, kDpThreads, 0, s>>>(a, st->vis); break;
        default: dp_reduce_adam_kernel<8><<<grid, kDpThreads, 0, s>>>(a, st->vis); break;
    }
    dp_wait_kernel<<<1, 32, 0, s>>>(a, 1, kDpWaitShards);
    engine_add_launches(4);
    DP_CUDA(cudaGetLastError());
    return MSPLAT_OK;
}

int msplat_dp_errors(int reset)
{
    std::lock_guard<std::mutex> lk(engine_mutex());
    if (engine_init()) return -1;
    DpState* st = nullptr;
    if (dp_state(&st)) return -1;
    int v = 0;
    const cudaStream_t s = engine_stream();
    if (cudaMemcpyAsync(&v, st->err, sizeof(int), cudaMemcpyDeviceToHost, s) != cudaSuccess ||
        cudaStreamSynchronize(s) != cudaSuccess)
        return -1;
    if (reset) cudaMemsetAsync(st->err, 0, sizeof(int), s);
    return v;
}

}  // extern "C"
