// msl_runtime.hpp -- threadgroup execution for the MSL shim (test
// infrastructure only).  A kernel launch is a set of threadgroups; each
// threadgroup runs its threads as fibers on one OS thread, threadgroups of a
// launch are spread over OpenMP threads.
#pragma once
#include <algorithm>
#include <functional>

#include "msl_shim.hpp"

namespace msl {

struct ThreadIds {
    uint3 gp;     // thread_position_in_grid
    uint3 tgid;   // threadgroup_position_in_grid
    uint3 lid;    // thread_position_in_threadgroup
    uint3 tpg;    // threads_per_threadgroup
    uint tr;      // thread_index_in_threadgroup
    uint lane;    // thread_index_in_simdgroup
    uint sgid;    // simdgroup_index_in_threadgroup
};

using ThreadFn = std::function<void(const ThreadIds&)>;

// Marks a new kernel launch (threadgroup arrays are refilled per launch).
void begin_launch();
// Runs one threadgroup's `n` threads to completion as fibers.
void run_threadgroup(const ThreadIds* ids, int n, const ThreadFn& fn);

// Uniform threadgroups: grid of `groups` threadgroups of `tg` threads, every
// thread launched (bounds are the kernels' own checks).
inline void dispatch_threadgroups(uint3 groups, uint3 tg, const ThreadFn& fn)
{
    begin_launch();
    const long long total = (long long)groups.x * groups.y * groups.z;
    const int n = (int)(tg.x * tg.y * tg.z);
#pragma omp parallel
    {
        std::vector<ThreadIds> ids(n);
#pragma omp for schedule(dynamic, 1)
        for (long long t = 0; t < total; t++) {
            uint3 g((uint)(t % groups.x), (uint)((t / groups.x) % groups.y),
                    (uint)(t / ((long long)groups.x * groups.y)));
            for (int k = 0; k < n; k++) {
                ThreadIds& d = ids[k];
                d.lid = uint3((uint)(k % tg.x), (uint)((k / tg.x) % tg.y), (uint)(k / (tg.x * tg.y)));
                d.tgid = g;
                d.tpg = tg;
                d.gp = uint3(g.x * tg.x + d.lid.x, g.y * tg.y + d.lid.y, g.z * tg.z + d.lid.z);
                d.tr = (uint)k;
                d.lane = (uint)(k & 31);
                d.sgid = (uint)(k >> 5);
            }
            run_threadgroup(ids.data(), n, fn);
        }
    }
}

// Independent threads (kernels without barriers or SIMD collectives).
template <class F>
inline void dispatch_threads_1d(uint n, F f)
{
#pragma omp parallel for schedule(static)
    for (long long i = 0; i < (long long)n; i++) f((uint)i);
}

template <class F>
inline void dispatch_threads_2d(uint w, uint h, F f)
{
#pragma omp parallel for schedule(static)
    for (long long j = 0; j < (long long)h; j++)
        for (uint i = 0; i < w; i++) f(uint2(i, (uint)j));
}

}  // namespace msl
