// kernels_sort.cu -- tile binning and the per-tile depth order by two
// global, stable LSD radix sorts.
//
// The reference bins each visible Gaussian's (tile, Gaussian) pairs into
// per-tile slots with atomics and sorts every tile's 64-bit keys (depth bits
// << 32 | id) by a bitonic network in threadgroup memory
// (scatter_to_prealloc_bins_kernel, msplat_metal.metal:2025-2059;
// bitonic_sort_per_tile_kernel, :2064-2138).  The same order follows from
// two stable sorts over the whole view, with no atomics on the keys and no
// ties to resolve:
//   1. the Gaussians by depth: keys depth bits (culled: 0xffffffff, last),
//      values the ids 0..N-1 in id order, four 8-bit passes; a stable sort
//      keeps equal depths in id order, so the result is the (depth, id)
//      order of the reference's keys;
//   2. the pairs, written in that order (rank r's tiles at the prefix sum
//      of the areas of ranks < r), by tile id, one or two 8-bit passes;
//      stability keeps each tile's pairs in (depth, id) order.
// Each pass is count / scan / scatter over tiles of 4096 keys: per-tile
// digit counts, one scan per digit over the tiles (offset of every
// (digit, tile) run in the output), then a stable scatter that ranks each
// tile's keys per digit in shared memory (warp match + per-warp counters,
// in input order) and writes them grouped by digit.  No block waits on
// another: at these sizes (1-6M Gaussians, 4-35M pairs, one or a few waves
// of blocks) a single-pass scheme's look-back chain costs more than the
// two extra launches.
#include <cuda_runtime.h>

#include <algorithm>
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

__device__ __forceinline__ long long os_items(const int* n_dev, long long n_host, long long cap)
{
    return n_dev ? min((long long)*n_dev, cap) : n_host;
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
// zeroed beforehand).  Each warp counts into its own shared copy (lanes of
// one warp with equal digits serialise only among themselves), then the
// block adds its copies into the global counts.
__global__ void __launch_bounds__(256)
depth_hist_kernel(int N, const float* __restrict__ depth, const int* __restrict__ radii,
                  unsigned* __restrict__ hist)
{
    __shared__ unsigned s[kOsWarps][4 * kOsRadix];
    const int warp = threadIdx.x >> 5;
    for (int i = threadIdx.x; i < kOsWarps * 4 * kOsRadix; i += blockDim.x) (&s[0][0])[i] = 0;
    __syncthreads();
    const DepthSource src{depth, radii};
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < N;
         i += (long long)gridDim.x * blockDim.x) {
        unsigned key, val;
        src.load(i, key, val);
#pragma unroll
        for (int p = 0; p < 4; p++) atomicAdd(&s[warp][p * kOsRadix + ((key >> (8 * p)) & 0xffu)], 1u);
    }
    __syncthreads();
    for (int i = threadIdx.x; i < 4 * kOsRadix; i += blockDim.x) {
        unsigned c = 0;
#pragma unroll
        for (int w = 0; w < kOsWarps; w++) c += s[w][i];
        if (c) atomicAdd(&hist[i], c);
    }
}

// Digit counts of each tile of 4096 keys: counts[d * ts + b] (ts = the
// tile stride of the counts array).
template <class Src>
__global__ void __launch_bounds__(kOsThreads)
digit_count_kernel(Src src, const int* __restrict__ n_dev, long long n_host, long long cap,
                   int shift, unsigned* __restrict__ counts, int ts)
{
    __shared__ unsigned s_whist[kOsWarps][kOsRadix];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const long long n = os_items(n_dev, n_host, cap);
    const long long tiles = (n + kOsTile - 1) / kOsTile;
    for (long long b = blockIdx.x; b < tiles; b += gridDim.x) {
        for (int i = lane; i < kOsRadix; i += 32) s_whist[warp][i] = 0;
        __syncwarp();
        const long long base = b * kOsTile + (long long)warp * (kOsItems * 32);
        unsigned key[kOsItems];
#pragma unroll
        for (int r = 0; r < kOsItems; r++) {   // every load in flight before any count
            const long long i = base + r * 32 + lane;
            unsigned val;
            key[r] = 0;
            if (i < n) src.load(i, key[r], val);
        }
#pragma unroll
        for (int r = 0; r < kOsItems; r++)
            if (base + r * 32 + lane < n) atomicAdd(&s_whist[warp][(key[r] >> shift) & 0xffu], 1u);
        __syncthreads();
        unsigned c = 0;
#pragma unroll
        for (int w = 0; w < kOsWarps; w++) c += s_whist[w][tid];
        counts[(size_t)tid * ts + b] = c;
        __syncthreads();
    }
}

// Output offset of every (digit, tile) run: block d scans digit d's counts
// over the tiles and adds the digit's base (exclusive scan of the pass's
// digit totals `hist`).
__global__ void __launch_bounds__(kOsThreads)
digit_scan_kernel(const unsigned* __restrict__ counts, unsigned* __restrict__ offs, int ts,
                  const unsigned* __restrict__ hist, const int* __restrict__ n_dev,
                  long long n_host, long long cap)
{
    __shared__ unsigned s_wsum[kOsWarps];
    __shared__ unsigned s_base;
    const int tid = threadIdx.x, d = blockIdx.x;
    const long long n = os_items(n_dev, n_host, cap);
    const long long tiles = (n + kOsTile - 1) / kOsTile;
    const unsigned excl = cta_excl_scan(hist[tid], s_wsum, nullptr);
    if (tid == d) s_base = excl;
    __syncthreads();
    unsigned run = s_base;
    const unsigned* c = counts + (size_t)d * ts;
    unsigned* o = offs + (size_t)d * ts;
    for (long long b0 = 0; b0 < tiles; b0 += kOsThreads) {
        const long long b = b0 + tid;
        const unsigned v = b < tiles ? c[b] : 0u;
        unsigned total = 0;
        const unsigned e = cta_excl_scan(v, s_wsum, &total);
        if (b < tiles) o[b] = run + e;
        run += total;
    }
}

// One stable LSD pass over digit (key >> shift) & 255 of n keys (n_dev
// when given, clamped to cap; else n_host), tile b's digit-d run starting
// at offs[d * ts + b].
template <class Src, class KeyT, bool WRITE_KEYS>
__global__ void __launch_bounds__(kOsThreads, 3)
digit_scatter_kernel(Src src, KeyT* __restrict__ keys_out, unsigned* __restrict__ vals_out,
                     const unsigned* __restrict__ offs, int ts, const int* __restrict__ n_dev,
                     long long n_host, long long cap, int shift)
{
    __shared__ unsigned s_whist[kOsWarps][kOsRadix];   // per-warp counts, then offsets
    __shared__ unsigned s_bexcl[kOsRadix];             // digit offsets inside this tile
    __shared__ unsigned s_gbase[kOsRadix];             // output position of the tile's digit
    __shared__ unsigned s_key[kOsTile];
    __shared__ unsigned s_val[kOsTile];
    __shared__ unsigned s_wsum[kOsWarps];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const unsigned lt = (1u << lane) - 1u;
    const long long n = os_items(n_dev, n_host, cap);
    const long long tiles = (n + kOsTile - 1) / kOsTile;
    for (long long b = blockIdx.x; b < tiles; b += gridDim.x) {
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
        s_gbase[tid] = offs[(size_t)tid * ts + b];
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
        // thread tid owns digit tid: the warps' offsets within the tile
        unsigned tot = 0;
#pragma unroll
        for (int w = 0; w < kOsWarps; w++) {
            const unsigned c = s_whist[w][tid];
            s_whist[w][tid] = tot;
            tot += c;
        }
        s_bexcl[tid] = cta_excl_scan(tot, s_wsum, nullptr);
        __syncthreads();   // every digit's tile offset before any thread reads it
        // the tile grouped by digit in shared memory, then written in runs
#pragma unroll
        for (int r = 0; r < kOsItems; r++) {
            if (base + r * 32 + lane >= n) continue;
            const unsigned d = (key[r] >> shift) & 0xffu;
            const unsigned lp = s_bexcl[d] + s_whist[warp][d] + rnk[r];
            if (lp >= (unsigned)kOsTile) continue;   // cannot happen: lp < the tile's count
            s_key[lp] = key[r];
            s_val[lp] = val[r];
        }
        __syncthreads();
        const int cnt = (int)min((long long)kOsTile, n - b * kOsTile);
        for (int i = tid; i < cnt; i += kOsThreads) {
            const unsigned k = s_key[i];
            const unsigned d = (k >> shift) & 0xffu;
            const unsigned pos = s_gbase[d] + ((unsigned)i - s_bexcl[d]);
            if (pos >= (unsigned long long)n) continue;   // only if the counts disagreed
            if (WRITE_KEYS) keys_out[pos] = (KeyT)k;
            vals_out[pos] = s_val[i];
        }
        __syncthreads();
    }
}

// Rect area of each rank (Gaussian ids[r] of the depth order; culled ones
// have none), summed per group of 32 consecutive ranks: sums[r / 32].
__device__ __forceinline__ unsigned rank_area(const unsigned* ids, const int* radii,
                                              const uint2* rect, long long r, long long N,
                                              unsigned& g, uint2& rc)
{
    g = 0;
    rc = make_uint2(0u, 0u);
    if (r >= N) return 0u;
    g = ids[r];
    if (radii[g] <= 0) return 0u;
    rc = rect[g];
    return ((rc.y & 0xffffu) - (rc.x & 0xffffu)) * ((rc.y >> 16) - (rc.x >> 16));
}

__global__ void __launch_bounds__(kOsThreads)
rank_area_kernel(int N, const unsigned* __restrict__ ids, const int* __restrict__ radii,
                 const uint2* __restrict__ rect, unsigned* __restrict__ sums)
{
    const long long r = (long long)blockIdx.x * kOsThreads + threadIdx.x;
    unsigned g;
    uint2 rc;
    const unsigned a = __reduce_add_sync(0xffffffffu, rank_area(ids, radii, rect, r, N, g, rc));
    if ((threadIdx.x & 31) == 0 && r < N) sums[r >> 5] = a;
}

// Exclusive prefix of sums[0, n) into offs, one CTA of 1024 threads: each
// thread adds up a contiguous run, the CTA scans the run totals, each
// thread writes its run's prefixes.
__global__ void __launch_bounds__(1024)
group_scan_kernel(const unsigned* __restrict__ sums, unsigned* __restrict__ offs, long long n)
{
    __shared__ unsigned s_w[32];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const long long per = (n + 1023) / 1024;
    const long long beg = min((long long)tid * per, n), end = min(beg + per, n);
    unsigned local = 0;
    for (long long i = beg; i < end; i++) local += sums[i];
    unsigned x = local;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const unsigned u = __shfl_up_sync(0xffffffffu, x, o);
        if (lane >= o) x += u;
    }
    if (lane == 31) s_w[warp] = x;
    __syncthreads();
    if (warp == 0) {
        const unsigned v = s_w[lane];
        unsigned y = v;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const unsigned u = __shfl_up_sync(0xffffffffu, y, o);
            if (lane >= o) y += u;
        }
        s_w[lane] = y - v;
    }
    __syncthreads();
    unsigned run = s_w[warp] + x - local;
    for (long long i = beg; i < end; i++) {
        offs[i] = run;
        run += sums[i];
    }
}

// The pairs of the depth-ordered Gaussians: rank r (Gaussian ids[r]) writes
// tile id (u16) and Gaussian id for each tile of its rect, row-major, at
// the prefix sum of the areas of the ranks before it.  One warp per group
// of 32 ranks (its first pair at offs[group]), the group's pairs dealt to
// the lanes 32 at a time; the tiles' low and high bytes are counted into
// hist[2][256] for the tile sort.  Pairs at or beyond cap are not written
// (nor counted): the scan of the tile counts has flagged the overflow.
__global__ void __launch_bounds__(kOsThreads)
pair_kernel(const StepParams* __restrict__ P, int N, const unsigned* __restrict__ ids,
            const int* __restrict__ radii, const uint2* __restrict__ rect,
            const unsigned* __restrict__ offs, unsigned short* __restrict__ pkey,
            unsigned* __restrict__ pval, unsigned* __restrict__ hist)
{
    __shared__ unsigned s_hist[2 * kOsRadix];
    const int tid = threadIdx.x, lane = tid & 31;
    for (int i = tid; i < 2 * kOsRadix; i += kOsThreads) s_hist[i] = 0;
    __syncthreads();
    const long long cap = P->capacity;
    const unsigned tx_n = (unsigned)P->tiles_x;
    const long long r = (long long)blockIdx.x * kOsThreads + tid;
    unsigned g;
    uint2 rc;
    const unsigned area = rank_area(ids, radii, rect, r, N, g, rc);
    unsigned incl = area;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const unsigned u = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += u;
    }
    const unsigned total = __shfl_sync(0xffffffffu, incl, 31);
    const unsigned long long off = r - lane < N ? offs[(r - lane) >> 5] : 0ull;
    for (unsigned p0 = 0; p0 < total; p0 += 32) {
        const unsigned pidx = p0 + lane;
        int owner = 0;
#pragma unroll
        for (int step = 16; step > 0; step >>= 1) {
            const unsigned probe = __shfl_sync(0xffffffffu, incl, owner + step - 1);
            if (probe <= pidx) owner += step;
        }
        const unsigned o_incl = __shfl_sync(0xffffffffu, incl, owner);
        const unsigned o_area = __shfl_sync(0xffffffffu, area, owner);
        const unsigned o_g = __shfl_sync(0xffffffffu, g, owner);
        const unsigned o_rx = __shfl_sync(0xffffffffu, rc.x, owner);
        const unsigned o_ry = __shfl_sync(0xffffffffu, rc.y, owner);
        if (pidx >= total) continue;
        const unsigned k = pidx - (o_incl - o_area);
        const unsigned x0 = o_rx & 0xffffu, y0 = o_rx >> 16;
        const unsigned w = (o_ry & 0xffffu) - x0;
        const unsigned tile = (y0 + k / w) * tx_n + x0 + k % w;
        const unsigned long long idx = off + pidx;
        if (idx < (unsigned long long)cap) {
            pkey[idx] = (unsigned short)tile;
            pval[idx] = o_g;
            atomicAdd(&s_hist[tile & 0xffu], 1u);
            atomicAdd(&s_hist[kOsRadix + (tile >> 8)], 1u);
        }
    }
    __syncthreads();
    for (int i = tid; i < 2 * kOsRadix; i += kOsThreads)
        if (s_hist[i]) atomicAdd(&hist[i], s_hist[i]);
}

namespace {

// Blocks of `kernel` (kOsThreads threads) resident on the current device at
// once, times two: the grid of the kernels that loop over tiles.  One
// lookup per kernel and device.
template <const void* (*KERNEL)()>
int loop_grid()
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
            blocks[d] = 2 * (sms > 0 ? sms : 148) * per;
        }) || cudaGetDevice(&dev) != cudaSuccess)
        return 2 * 148;
    return blocks[dev];
}

template <class Src>
const void* count_ptr() { return (const void*)digit_count_kernel<Src>; }
template <class Src, class KeyT, bool WK>
const void* scatter_ptr() { return (const void*)digit_scatter_kernel<Src, KeyT, WK>; }

int grid_for(long long max_items, int per_launch)
{
    const long long tiles = (max_items + kOsTile - 1) / kOsTile;
    return (int)std::max(1LL, std::min(tiles, (long long)per_launch));
}

// One LSD pass: counts, per-digit scan, scatter.  counts / offs: the two
// halves of SortBuffers::status, ts tiles each per digit.
template <class Src, class KeyT, bool WK>
void launch_pass(Src src, KeyT* keys_out, unsigned* vals_out, const unsigned* hist,
                 const SortBuffers& S, int ts, const int* n_dev, long long n_host, long long cap,
                 long long max_items, int shift, cudaStream_t s)
{
    unsigned* counts = reinterpret_cast<unsigned*>(S.status);
    unsigned* offs = counts + (size_t)kOsRadix * ts;
    digit_count_kernel<Src><<<grid_for(max_items, loop_grid<count_ptr<Src>>()), kOsThreads, 0, s>>>(
        src, n_dev, n_host, cap, shift, counts, ts);
    digit_scan_kernel<<<kOsRadix, kOsThreads, 0, s>>>(counts, offs, ts, hist, n_dev, n_host, cap);
    digit_scatter_kernel<Src, KeyT, WK>
        <<<grid_for(max_items, loop_grid<scatter_ptr<Src, KeyT, WK>>()), kOsThreads, 0, s>>>(
            src, keys_out, vals_out, offs, ts, n_dev, n_host, cap, shift);
}

}  // namespace

// Length (in 64-bit words) of SortBuffers::status: the count and offset
// arrays of the passes, 256 u32 each per tile of 4096 keys of the larger
// of the two sorts.
long long sort_status_words(long long N, long long cap)
{
    return std::max((N + kOsTile - 1) / kOsTile, (cap + kOsTile - 1) / kOsTile) * kOsRadix;
}

// Depth sort, pair generation and tile sort; the sorted Gaussian ids go to
// B.sorted_ids.  S.ctrl (histograms) was zeroed by the scan of the tile
// counts earlier on the stream.  Returns the kernels launched.
int launch_bin_sort(const StepParams* P, int N, int num_tiles, long long cap, const Buffers& B,
                    cudaStream_t s)
{
    if (N <= 0) return 0;
    const SortBuffers& S = B.sort;
    const int ts = (int)(sort_status_words(N, cap) / kOsRadix);
    unsigned* hist_d = S.ctrl + kSortCtrlHistDepth;
    unsigned* hist_p = S.ctrl + kSortCtrlHistPair;
    const int hgrid = std::min((N + 255) / 256, 2 * 148);
    depth_hist_kernel<<<hgrid, 256, 0, s>>>(N, B.proj.depth, B.proj.radii, hist_d);
    // four passes over the depth keys: depth -> b -> a -> b -> a (values only last)
    launch_pass<DepthSource, unsigned, true>(DepthSource{B.proj.depth, B.proj.radii}, S.dkey_b,
                                             S.dval_b, hist_d, S, ts, nullptr, N, N, N, 0, s);
    launch_pass<ArraySource<unsigned>, unsigned, true>(ArraySource<unsigned>{S.dkey_b, S.dval_b},
                                                       S.dkey_a, S.dval_a, hist_d + 256, S, ts,
                                                       nullptr, N, N, N, 8, s);
    launch_pass<ArraySource<unsigned>, unsigned, true>(ArraySource<unsigned>{S.dkey_a, S.dval_a},
                                                       S.dkey_b, S.dval_b, hist_d + 512, S, ts,
                                                       nullptr, N, N, N, 16, s);
    launch_pass<ArraySource<unsigned>, unsigned, false>(ArraySource<unsigned>{S.dkey_b, S.dval_b},
                                                        nullptr, S.dval_a, hist_d + 768, S, ts,
                                                        nullptr, N, N, N, 24, s);
    // pairs in depth order: area sums per 32 ranks (in the counts half of
    // status), their prefix (in the offsets half), then the pairs
    unsigned* sums = reinterpret_cast<unsigned*>(S.status);
    unsigned* goffs = sums + (size_t)kOsRadix * ts;
    const int rgrid = (N + kOsThreads - 1) / kOsThreads;
    rank_area_kernel<<<rgrid, kOsThreads, 0, s>>>(N, S.dval_a, B.proj.radii, B.proj.rect, sums);
    group_scan_kernel<<<1, 1024, 0, s>>>(sums, goffs, ((long long)N + 31) / 32);
    pair_kernel<<<rgrid, kOsThreads, 0, s>>>(P, N, S.dval_a, B.proj.radii, B.proj.rect, goffs,
                                             S.pkey_a, S.pval_a, hist_p);
    // stable sort of the pairs by tile id: one pass per byte of the tile ids
    const int* n_dev = B.tile_offset + num_tiles;
    unsigned* ids = reinterpret_cast<unsigned*>(B.sorted_ids);
    if (num_tiles <= kOsRadix) {
        launch_pass<ArraySource<unsigned short>, unsigned short, false>(
            ArraySource<unsigned short>{S.pkey_a, S.pval_a}, nullptr, ids, hist_p, S, ts, n_dev, 0,
            cap, cap, 0, s);
        return 1 + 12 + 3 + 3;
    }
    launch_pass<ArraySource<unsigned short>, unsigned short, true>(
        ArraySource<unsigned short>{S.pkey_a, S.pval_a}, S.pkey_b, S.pval_b, hist_p, S, ts, n_dev, 0,
        cap, cap, 0, s);
    launch_pass<ArraySource<unsigned short>, unsigned short, false>(
        ArraySource<unsigned short>{S.pkey_b, S.pval_b}, nullptr, ids, hist_p + kOsRadix, S, ts,
        n_dev, 0, cap, cap, 8, s);
    return 1 + 12 + 3 + 6;
}

}  // namespace msp
