// kernels_sort.cu -- tile binning and the per-tile depth order by two
// global, stable, one-sweep radix sorts.
//
// The reference bins each visible Gaussian's (tile, Gaussian) pairs into
// per-tile slots with atomics and sorts every tile's 64-bit keys (depth bits
// << 32 | id) by a bitonic network in threadgroup memory
// (scatter_to_prealloc_bins_kernel, msplat_metal.metal:2025-2059;
// bitonic_sort_per_tile_kernel, :2064-2138).  The same order follows from
// two stable sorts over the whole view, with no atomics and no ties to
// resolve:
//   1. the Gaussians by depth: keys depth bits (culled: 0xffffffff, last),
//      values the ids 0..N-1 in id order, four 8-bit LSD passes; a stable
//      sort keeps equal depths in id order, so the result is the
//      (depth, id) order of the reference's keys;
//   2. the pairs, written in that order (rank r's tiles at the prefix sum
//      of the areas of ranks < r), by tile id, one or two 8-bit LSD passes;
//      stability keeps each tile's pairs in (depth, id) order.
// Each pass is one kernel: a block takes the next 4096 keys by ticket, ranks
// them per 8-bit digit in shared memory (warp-level match + per-warp
// counters, in input order), publishes its digit counts, finds the counts
// of all earlier blocks by decoupled look-back over their published words,
// and writes its keys grouped by digit (coalesced runs).  The digit totals
// of the whole pass come from one histogram read made before.  Every
// look-back wait is bounded by %globaltimer; a block that gives up sets
// kErrSortTimeout, publishes a word anyway (so no later block waits on it)
// and writes nothing.
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <cstdint>
#include <mutex>

#include "engine.h"
#include "msp_math.cuh"

namespace msp {

constexpr int kOsThreads = 256;
constexpr int kOsWarps = kOsThreads / 32;
constexpr int kOsItems = 16;                         // keys per thread
constexpr int kOsTile = kOsThreads * kOsItems;       // keys per block tile
constexpr int kOsRadix = 256;
constexpr unsigned kOsNone = 256;                    // digit of a padding slot
constexpr unsigned long long kOsLookbackNs = 2000000000ull;   // 2 s

// Published words: flag [63:62] (1 = this block's counts, 2 = inclusive
// prefix), epoch [61:30] (the launch), count [29:0].
constexpr unsigned long long kOsAgg = 1ull << 62, kOsPrefix = 2ull << 62;
__device__ __forceinline__ unsigned long long os_word(unsigned long long flag, unsigned epoch,
                                                      unsigned long long count)
{
    return flag | ((unsigned long long)epoch << 30) | (count & ((1ull << 30) - 1));
}
__device__ __forceinline__ unsigned os_epoch(unsigned long long w)
{
    return (unsigned)(w >> 30);
}
__device__ __forceinline__ unsigned long long os_count(unsigned long long w)
{
    return w & ((1ull << 30) - 1);
}

__device__ __forceinline__ unsigned long long os_now()
{
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// Exclusive prefix over the CTA of one value per thread (kOsThreads).
__device__ __forceinline__ unsigned cta_excl_scan(unsigned v, unsigned* s_wsum, unsigned* total)
{
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    unsigned x = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const unsigned u = __shfl_up_sync(0xffffffffu, x, o);
        if (lane >= o) x += u;
    }
    if (lane == 31) s_wsum[warp] = x;
    __syncthreads();
    unsigned before = 0, all = 0;
#pragma unroll
    for (int w = 0; w < kOsWarps; w++) {
        const unsigned s = s_wsum[w];
        before += w < warp ? s : 0u;
        all += s;
    }
    __syncthreads();
    if (total) *total = all;
    return before + x - v;
}

__device__ __forceinline__ bool os_ready(unsigned long long w, unsigned epoch)
{
    return os_epoch(w) == epoch && (w >> 62) != 0;
}

// Decoupled look-back by one thread: the sum of `slot` over every block
// before `b`, from words published under `epoch`, reading kOsWindow
// predecessors per round (their loads in flight together: every block of a
// wave starts at once, so the nearest inclusive prefix can be far back).
// False when a wait ran out.
constexpr int kOsWindow = 8;
__device__ __forceinline__ bool os_lookback(const unsigned long long* status, long long b,
                                            int stride, int slot, unsigned epoch,
                                            unsigned long long& excl)
{
    excl = 0;
    long long j = b - 1;   // nearest predecessor not yet summed
    unsigned long long t0 = 0;
    while (j >= 0) {
        unsigned long long w[kOsWindow];
#pragma unroll
        for (int k = 0; k < kOsWindow; k++)
            w[k] = j - k >= 0 ? *reinterpret_cast<const volatile unsigned long long*>(
                                    status + (j - k) * stride + slot)
                              : os_word(kOsPrefix, epoch, 0);
        int used = 0;
        bool done = false, stalled = false;
#pragma unroll
        for (int k = 0; k < kOsWindow; k++) {
            if (done || stalled) continue;
            if (!os_ready(w[k], epoch)) {
                stalled = true;
                continue;
            }
            excl += os_count(w[k]);
            used++;
            done = (w[k] & kOsPrefix) != 0;
        }
        if (done) return true;
        j -= used;
        if (used == 0) {
            const unsigned long long now = os_now();
            if (t0 == 0) t0 = now;
            else if (now - t0 > kOsLookbackNs) return false;
        }
    }
    return true;
}

// The same for a single value per block, by a whole warp: lane k reads
// predecessor j - k, 32 per round.  Every lane returns the same result.
__device__ __forceinline__ bool os_lookback_warp(const unsigned long long* status, long long b,
                                                 unsigned epoch, unsigned long long& excl)
{
    const int lane = threadIdx.x & 31;
    excl = 0;
    long long j = b - 1;
    unsigned long long t0 = 0;
    while (j >= 0) {
        const long long idx = j - lane;
        const unsigned long long w =
            idx >= 0 ? *reinterpret_cast<const volatile unsigned long long*>(status + idx)
                     : os_word(kOsPrefix, epoch, 0);
        const bool ready = os_ready(w, epoch);
        const unsigned notready = __ballot_sync(0xffffffffu, !ready);
        const unsigned prefix = __ballot_sync(0xffffffffu, ready && (w & kOsPrefix) != 0);
        const int fnr = notready ? __ffs(notready) - 1 : 32;
        const int fp = prefix ? __ffs(prefix) - 1 : 32;
        const int take = fp < fnr ? fp + 1 : fnr;   // lanes [0, take) are summed
        unsigned long long c = lane < take ? os_count(w) : 0ull;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) c += __shfl_xor_sync(0xffffffffu, c, o);
        excl += c;
        if (fp < fnr) return true;
        j -= take;
        if (take == 0) {
            const unsigned long long now = os_now();
            if (t0 == 0) t0 = now;
            else if (now - t0 > kOsLookbackNs) return false;
        }
    }
    return true;
}

__device__ __forceinline__ void os_publish(unsigned long long* status, long long b, int stride,
                                           int slot, unsigned long long word)
{
    *reinterpret_cast<volatile unsigned long long*>(status + b * stride + slot) = word;
}

// ---- sources of the first pass of each sort --------------------------------

// Depth sort input: key = depth bits (radius > 0; depths of visible
// Gaussians are positive, so their bits order as the floats), else
// 0xffffffff; value = the Gaussian id.
struct DepthSource {
    const float* depth;
    const int* radii;
    __device__ __forceinline__ void load(long long i, unsigned& key, unsigned& val) const
    {
        key = radii[i] > 0 ? __float_as_uint(depth[i]) : 0xffffffffu;
        val = (unsigned)i;
    }
};

template <class K>
struct ArraySource {
    const K* keys;
    const unsigned* vals;
    __device__ __forceinline__ void load(long long i, unsigned& key, unsigned& val) const
    {
        key = keys[i];
        val = vals[i];
    }
};

// Histograms of the four 8-bit digits of the depth keys (hist[4][256],
// zeroed beforehand).
__global__ void __launch_bounds__(256)
depth_hist_kernel(int N, const float* __restrict__ depth, const int* __restrict__ radii,
                  unsigned* __restrict__ hist)
{
    __shared__ unsigned s[4 * kOsRadix];
    for (int i = threadIdx.x; i < 4 * kOsRadix; i += blockDim.x) s[i] = 0;
    __syncthreads();
    const DepthSource src{depth, radii};
    const int lane = threadIdx.x & 31;
    for (long long base = (long long)blockIdx.x * blockDim.x; base < N;
         base += (long long)gridDim.x * blockDim.x) {
        const long long i = base + threadIdx.x;
        unsigned key = 0, val = 0;
        const bool ok = i < N;
        if (ok) src.load(i, key, val);
#pragma unroll
        for (int p = 0; p < 4; p++) {
            const unsigned d = ok ? (key >> (8 * p)) & 0xffu : kOsNone;
            const unsigned peers = __match_any_sync(0xffffffffu, d);
            if (ok && lane == __ffs(peers) - 1) atomicAdd(&s[p * kOsRadix + d], __popc(peers));
        }
    }
    __syncthreads();
    for (int i = threadIdx.x; i < 4 * kOsRadix; i += blockDim.x)
        if (s[i]) atomicAdd(&hist[i], s[i]);
}

// One stable LSD pass over digit (key >> shift) & 255 of n keys (n_dev
// when given, clamped to cap; else n_host).  Persistent: each block takes
// tiles by ticket until none are left.
template <class Src, class KeyT, bool WRITE_KEYS>
__global__ void __launch_bounds__(kOsThreads, 3)
onesweep_kernel(Src src, KeyT* __restrict__ keys_out, unsigned* __restrict__ vals_out,
                const unsigned* __restrict__ hist, unsigned long long* __restrict__ status,
                unsigned* __restrict__ ticket, const int* __restrict__ n_dev, long long n_host,
                long long cap, int shift, unsigned epoch, int* __restrict__ err)
{
    __shared__ unsigned s_whist[kOsWarps][kOsRadix];   // per-warp counts, then offsets
    __shared__ unsigned s_gexcl[kOsRadix];             // digit offsets of the whole pass
    __shared__ unsigned s_bexcl[kOsRadix];             // digit offsets inside this tile
    __shared__ unsigned s_gbase[kOsRadix];             // output position of the tile's digit
    __shared__ unsigned s_key[kOsTile];
    __shared__ unsigned s_val[kOsTile];
    __shared__ unsigned s_wsum[kOsWarps];
    __shared__ long long s_tile;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const unsigned lt = (1u << lane) - 1u;
    const long long n = n_dev ? min((long long)*n_dev, cap) : n_host;
    s_gexcl[tid] = cta_excl_scan(hist[tid], s_wsum, nullptr);
    for (;;) {
        if (tid == 0) s_tile = (long long)atomicAdd(ticket, 1u);
        __syncthreads();
        const long long b = s_tile;
        if (b * kOsTile >= n) break;
        const long long base = b * kOsTile + (long long)warp * (kOsItems * 32);
        unsigned key[kOsItems], val[kOsItems], rnk[kOsItems];
#pragma unroll
        for (int r = 0; r < kOsItems; r++) {
            const long long i = base + r * 32 + lane;
            key[r] = 0;
            val[r] = 0;
            if (i < n) src.load(i, key[r], val[r]);
        }
        for (int i = lane; i < kOsRadix; i += 32) s_whist[warp][i] = 0;
        __syncwarp();
        // ranks among the warp's keys of the same digit, in input order
#pragma unroll
        for (int r = 0; r < kOsItems; r++) {
            const bool ok = base + r * 32 + lane < n;
            const unsigned d = ok ? (key[r] >> shift) & 0xffu : kOsNone;
            const unsigned peers = __match_any_sync(0xffffffffu, d);
            rnk[r] = ok ? s_whist[warp][d] + __popc(peers & lt) : 0u;
            __syncwarp();
            if (ok && lane == __ffs(peers) - 1) s_whist[warp][d] += __popc(peers);
            __syncwarp();
        }
        __syncthreads();
        // thread tid owns digit tid: warp offsets, tile count, publication
        unsigned tot = 0;
#pragma unroll
        for (int w = 0; w < kOsWarps; w++) {
            const unsigned c = s_whist[w][tid];
            s_whist[w][tid] = tot;
            tot += c;
        }
        os_publish(status, b, kOsRadix, tid, os_word(b == 0 ? kOsPrefix : kOsAgg, epoch, tot));
        s_bexcl[tid] = cta_excl_scan(tot, s_wsum, nullptr);
        unsigned long long excl = 0;
        bool ok = true;
        if (b > 0) {
            ok = os_lookback(status, b, kOsRadix, tid, epoch, excl);
            os_publish(status, b, kOsRadix, tid, os_word(kOsPrefix, epoch, excl + tot));
        }
        s_gbase[tid] = s_gexcl[tid] + (unsigned)excl;
        if (__syncthreads_or(!ok)) {
            if (tid == 0) atomicOr(err, kErrSortTimeout);
            continue;
        }
        // the tile grouped by digit in shared memory, then written in runs
#pragma unroll
        for (int r = 0; r < kOsItems; r++) {
            if (base + r * 32 + lane >= n) continue;
            const unsigned d = (key[r] >> shift) & 0xffu;
            const unsigned lp = s_bexcl[d] + s_whist[warp][d] + rnk[r];
            s_key[lp] = key[r];
            s_val[lp] = val[r];
        }
        __syncthreads();
        const int cnt = (int)min((long long)kOsTile, n - b * kOsTile);
        for (int i = tid; i < cnt; i += kOsThreads) {
            const unsigned k = s_key[i];
            const unsigned d = (k >> shift) & 0xffu;
            const unsigned pos = s_gbase[d] + ((unsigned)i - s_bexcl[d]);
            if (pos >= (unsigned long long)n) continue;   // only if the histogram disagreed
            if (WRITE_KEYS) keys_out[pos] = (KeyT)k;
            vals_out[pos] = s_val[i];
        }
        __syncthreads();
    }
}

// The pairs of the depth-ordered Gaussians: rank r (Gaussian ids[r]) writes
// tile id (u16) and Gaussian id for each tile of its rect, row-major, at
// the prefix sum of the areas of the ranks before it (decoupled look-back
// over blocks of 4096 ranks); tiles' low and high bytes are counted into
// hist[2][256] for the tile sort.  Pairs at or beyond cap are not written
// (nor counted): the scan of the tile counts has flagged the overflow.
__global__ void __launch_bounds__(kOsThreads)
pair_kernel(const StepParams* __restrict__ P, int N, const unsigned* __restrict__ ids,
            const int* __restrict__ radii, const uint2* __restrict__ rect,
            unsigned short* __restrict__ pkey, unsigned* __restrict__ pval,
            unsigned* __restrict__ hist, unsigned long long* __restrict__ status,
            unsigned* __restrict__ ticket, unsigned epoch, int* __restrict__ err)
{
    __shared__ unsigned s_hist[2 * kOsRadix];
    __shared__ unsigned s_wsum[kOsWarps];
    __shared__ long long s_tile;
    __shared__ unsigned long long s_base;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    for (int i = tid; i < 2 * kOsRadix; i += kOsThreads) s_hist[i] = 0;
    const long long cap = P->capacity;
    const int tx_n = P->tiles_x;
    for (;;) {
        if (tid == 0) s_tile = (long long)atomicAdd(ticket, 1u);
        __syncthreads();
        const long long b = s_tile;
        if (b * kOsTile >= N) break;
        const long long base = b * kOsTile + (long long)warp * (kOsItems * 32);
        // areas of the warp's 512 ranks (rank-major over lanes, then groups)
        unsigned area[kOsItems];
        unsigned wsum = 0;
#pragma unroll
        for (int q = 0; q < kOsItems; q++) {
            const long long r = base + q * 32 + lane;
            area[q] = 0;
            if (r < N) {
                const unsigned g = ids[r];
                if (radii[g] > 0) {
                    const uint2 rc = rect[g];
                    area[q] = ((rc.y & 0xffffu) - (rc.x & 0xffffu)) * ((rc.y >> 16) - (rc.x >> 16));
                }
            }
            wsum += __reduce_add_sync(0xffffffffu, area[q]);
        }
        unsigned btotal = 0;
        const unsigned wex = cta_excl_scan(lane == 0 ? wsum : 0u, s_wsum, &btotal);
        const unsigned warp_base = __shfl_sync(0xffffffffu, wex, 0);
        if (warp == 0) {
            if (lane == 0)
                os_publish(status, b, 1, 0, os_word(b == 0 ? kOsPrefix : kOsAgg, epoch, btotal));
            unsigned long long excl = 0;
            bool ok = true;
            if (b > 0) {
                ok = os_lookback_warp(status, b, epoch, excl);
                if (lane == 0) os_publish(status, b, 1, 0, os_word(kOsPrefix, epoch, excl + btotal));
            }
            if (lane == 0) {
                if (!ok) atomicOr(err, kErrSortTimeout);
                s_base = ok ? excl : ~0ull;
            }
        }
        __syncthreads();
        const unsigned long long bbase = s_base;
        if (bbase == ~0ull) continue;
        unsigned long long off = bbase + warp_base;
        // deal each group's pairs to the lanes, 32 at a time
#pragma unroll 1
        for (int q = 0; q < kOsItems; q++) {
            unsigned incl = area[q];
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const unsigned u = __shfl_up_sync(0xffffffffu, incl, o);
                if (lane >= o) incl += u;
            }
            const unsigned total = __shfl_sync(0xffffffffu, incl, 31);
            const long long r = base + q * 32 + lane;
            const unsigned g = r < N ? ids[r] : 0u;
            const uint2 rc = area[q] ? rect[g] : make_uint2(0u, 0u);
            for (unsigned p0 = 0; p0 < total; p0 += 32) {
                const unsigned pidx = p0 + lane;
                int owner = 0;
#pragma unroll
                for (int step = 16; step > 0; step >>= 1) {
                    const unsigned probe = __shfl_sync(0xffffffffu, incl, owner + step - 1);
                    if (probe <= pidx) owner += step;
                }
                const unsigned o_incl = __shfl_sync(0xffffffffu, incl, owner);
                const unsigned o_area = __shfl_sync(0xffffffffu, area[q], owner);
                const unsigned o_g = __shfl_sync(0xffffffffu, g, owner);
                const unsigned o_rx = __shfl_sync(0xffffffffu, rc.x, owner);
                const unsigned o_ry = __shfl_sync(0xffffffffu, rc.y, owner);
                if (pidx >= total) continue;
                const unsigned k = pidx - (o_incl - o_area);
                const unsigned x0 = o_rx & 0xffffu, y0 = o_rx >> 16;
                const unsigned w = (o_ry & 0xffffu) - x0;
                const unsigned tile = (y0 + k / w) * (unsigned)tx_n + x0 + k % w;
                const unsigned long long idx = off + pidx;
                if (idx < (unsigned long long)cap) {
                    pkey[idx] = (unsigned short)tile;
                    pval[idx] = o_g;
                    atomicAdd(&s_hist[tile & 0xffu], 1u);
                    atomicAdd(&s_hist[kOsRadix + (tile >> 8)], 1u);
                }
            }
            off += total;
        }
    }
    __syncthreads();
    for (int i = tid; i < 2 * kOsRadix; i += kOsThreads)
        if (s_hist[i]) atomicAdd(&hist[i], s_hist[i]);
}

namespace {

std::atomic<unsigned> g_epoch{8};

// Blocks of `kernel` (kOsThreads threads) resident on the current device at
// once: the persistent grid size.  One lookup per kernel and device.
template <const void* (*KERNEL)()>
int resident_blocks()
{
    static std::once_flag once[kMaxDeviceSlots];
    static int blocks[kMaxDeviceSlots];
    int dev = 0;
    if (!once_per_device(once, [](int d) {
            int sms = 0, per = 0;
            cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, d);
            if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per, KERNEL(), kOsThreads, 0) !=
                    cudaSuccess ||
                per < 1)
                per = 1;
            blocks[d] = (sms > 0 ? sms : 148) * per;
        }) || cudaGetDevice(&dev) != cudaSuccess)
        return 148;
    return blocks[dev];
}

template <class Src, class KeyT, bool WK>
const void* onesweep_ptr() { return (const void*)onesweep_kernel<Src, KeyT, WK>; }
const void* pair_ptr() { return (const void*)pair_kernel; }

template <class Src, class KeyT, bool WK>
void launch_pass(Src src, KeyT* keys_out, unsigned* vals_out, const unsigned* hist,
                 const SortBuffers& S, int ticket, const int* n_dev, long long n_host,
                 long long cap, long long max_items, int shift, unsigned epoch, int* err,
                 cudaStream_t s)
{
    const long long tiles = (max_items + kOsTile - 1) / kOsTile;
    const int grid = (int)std::max(
        1LL, std::min(tiles, (long long)resident_blocks<onesweep_ptr<Src, KeyT, WK>>()));
    onesweep_kernel<Src, KeyT, WK><<<grid, kOsThreads, 0, s>>>(
        src, keys_out, vals_out, hist, S.status, S.ctrl + ticket, n_dev, n_host, cap, shift, epoch,
        err);
}

}  // namespace

long long sort_status_words(long long N, long long cap)
{
    return std::max((N + kOsTile - 1) / kOsTile, (cap + kOsTile - 1) / kOsTile) * kOsRadix;
}

// Depth sort, pair generation and tile sort; the sorted Gaussian ids go to
// B.sorted_ids.  S.ctrl (tickets and histograms) was zeroed by the scan of
// the tile counts earlier on the stream.  Returns the kernels launched.
int launch_bin_sort(const StepParams* P, int N, int num_tiles, long long cap, const Buffers& B,
                    cudaStream_t s)
{
    if (N <= 0) return 0;
    const SortBuffers& S = B.sort;
    const unsigned epoch = g_epoch.fetch_add(8u);
    unsigned* hist_d = S.ctrl + kSortCtrlHistDepth;
    unsigned* hist_p = S.ctrl + kSortCtrlHistPair;
    const int hgrid = std::min((N + 255) / 256, 2 * 148);
    depth_hist_kernel<<<hgrid, 256, 0, s>>>(N, B.proj.depth, B.proj.radii, hist_d);
    // four passes over the depth keys: a -> b -> a -> b -> a (values only last)
    launch_pass<DepthSource, unsigned, true>(DepthSource{B.proj.depth, B.proj.radii}, S.dkey_b,
                                             S.dval_b, hist_d, S, 0, nullptr, N, N, N, 0,
                                             epoch + 0, B.err, s);
    launch_pass<ArraySource<unsigned>, unsigned, true>(ArraySource<unsigned>{S.dkey_b, S.dval_b},
                                                       S.dkey_a, S.dval_a, hist_d + 256, S, 1,
                                                       nullptr, N, N, N, 8, epoch + 1, B.err, s);
    launch_pass<ArraySource<unsigned>, unsigned, true>(ArraySource<unsigned>{S.dkey_a, S.dval_a},
                                                       S.dkey_b, S.dval_b, hist_d + 512, S, 2,
                                                       nullptr, N, N, N, 16, epoch + 2, B.err, s);
    launch_pass<ArraySource<unsigned>, unsigned, false>(ArraySource<unsigned>{S.dkey_b, S.dval_b},
                                                        nullptr, S.dval_a, hist_d + 768, S, 3,
                                                        nullptr, N, N, N, 24, epoch + 3, B.err, s);
    // pairs in depth order
    {
        const long long tiles = (N + kOsTile - 1) / kOsTile;
        const int grid = (int)std::max(1LL, std::min(tiles, (long long)resident_blocks<pair_ptr>()));
        pair_kernel<<<grid, kOsThreads, 0, s>>>(P, N, S.dval_a, B.proj.radii, B.proj.rect,
                                                S.pkey_a, S.pval_a, hist_p, S.status,
                                                S.ctrl + 4, epoch + 4, B.err);
    }
    // stable sort of the pairs by tile id: one pass per byte of the tile ids
    const int* n_dev = B.tile_offset + num_tiles;
    if (num_tiles <= kOsRadix) {
        launch_pass<ArraySource<unsigned short>, unsigned short, false>(
            ArraySource<unsigned short>{S.pkey_a, S.pval_a}, nullptr,
            reinterpret_cast<unsigned*>(B.sorted_ids), hist_p, S, 5, n_dev, 0, cap, cap, 0,
            epoch + 5, B.err, s);
        return 7;
    }
    launch_pass<ArraySource<unsigned short>, unsigned short, true>(
        ArraySource<unsigned short>{S.pkey_a, S.pval_a}, S.pkey_b, S.pval_b, hist_p, S, 5, n_dev,
        0, cap, cap, 0, epoch + 5, B.err, s);
    launch_pass<ArraySource<unsigned short>, unsigned short, false>(
        ArraySource<unsigned short>{S.pkey_b, S.pval_b}, nullptr,
        reinterpret_cast<unsigned*>(B.sorted_ids), hist_p + kOsRadix, S, 6, n_dev, 0, cap, cap, 8,
        epoch + 6, B.err, s);
    return 8;
}

}  // namespace msp
