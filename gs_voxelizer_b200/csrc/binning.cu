// Binning: (tile, gaussian) pairs ordered by tile id, then gaussian id.
//
// The reference (gs_voxelizer/cuda/bin_and_sort_gaussians.cu:11-62,
// bindings.cu:261-360) writes one key per pair in gaussian order and runs a
// stable 32-bit CUB radix sort, so inside each tile the gaussian ids come out
// ascending. Here the same order is produced with a counting sort keyed by
// tile id, which needs no key bits beyond the tile count:
//   1. count:   per-tile pair counts (atomics, order independent)
//   2. scan:    exclusive prefix sum over tiles -> tile_bins, per-tile cursors
//   3. scatter: each pair claims a slot in its tile's range (atomics; the order
//               inside a tile is arbitrary at this point)
//   4. sort:    every tile's segment is sorted ascending by gaussian id, which
//               restores the stable-sort order exactly (ids are unique inside
//               a tile). Segments of <= 256 ids are sorted in registers by one
//               warp, <= 16384 in shared memory by one CTA, larger ones by a
//               single-CTA radix sort through a global temporary.
// Pair expansion (steps 1 and 3) is load-balanced across a warp: the warp's 32
// Gaussians' tile boxes are flattened with a warp scan and each lane takes
// every 32nd pair, so a Gaussian covering 100 tiles does not stall its warp.
#include "common.cuh"

namespace gsv {
namespace {

constexpr int kScanThreads = 256;
constexpr int kScanItems = 2;
constexpr int kScanTile = kScanThreads * kScanItems;  // 512

struct Box {
    int x0, y0, z0, nx, ny, nz;
};

// Gaussian i's tile box clipped to the slab's tile-z range.
__device__ __forceinline__ Box load_box(const int *tmin, const int *tmax,
                                        int i, int tz0, int tz1) {
    Box b;
    b.x0 = tmin[3 * i + 0];
    b.y0 = tmin[3 * i + 1];
    const int z0 = max(tmin[3 * i + 2], tz0);
    const int z1 = min(tmax[3 * i + 2], tz1);
    b.z0 = z0;
    b.nx = max(0, tmax[3 * i + 0] - b.x0);
    b.ny = max(0, tmax[3 * i + 1] - b.y0);
    b.nz = max(0, z1 - z0);
    return b;
}

enum ExpandMode { kCount = 0, kScatter = 1 };

// mode kCount:   counts[tile] += 1 for every pair
// mode kScatter: ids[cursor[tile]++] = gaussian for every pair
// Gaussians are taken in the order `order` gives (all n of them), or in
// index order when it is null.
template <int MODE>
__global__ void __launch_bounds__(256)
expand_pairs_kernel(int n, const int *__restrict__ tmin,
                    const int *__restrict__ tmax, int Tx, int Ty, int tz0,
                    int tz1, int *__restrict__ counter,
                    int *__restrict__ ids_out, long long capacity,
                    int *__restrict__ error_flag,
                    const int *__restrict__ order) {
    const int lane = threadIdx.x & 31;
    const long long warp_global =
        ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const long long warps_total = ((long long)gridDim.x * blockDim.x) >> 5;
    for (long long w = warp_global; w * 32 < n; w += warps_total) {
        const long long gi = w * 32 + lane;
        Box b = {0, 0, 0, 0, 0, 0};
        int gid = 0;
        if (gi < n) {
            gid = order ? order[gi] : (int)gi;
            b = load_box(tmin, tmax, gid, tz0, tz1);
        }
        const int cnt = b.nx * b.ny * b.nz;
        const int incl = warp_inclusive_scan(cnt);
        const int excl = incl - cnt;
        const int total = __shfl_sync(0xffffffffu, incl, 31);
        for (int base = 0; base < total; base += 32) {
            const int k = base + lane;
            // owner = number of lanes whose inclusive end is <= k
            int owner = 0;
#pragma unroll
            for (int step = 16; step >= 1; step >>= 1) {
                const int probe_end =
                    __shfl_sync(0xffffffffu, incl, owner + step - 1);
                if (probe_end <= k) owner += step;
            }
            owner = min(owner, 31);
            const int o_excl = __shfl_sync(0xffffffffu, excl, owner);
            const int o_x0 = __shfl_sync(0xffffffffu, b.x0, owner);
            const int o_y0 = __shfl_sync(0xffffffffu, b.y0, owner);
            const int o_z0 = __shfl_sync(0xffffffffu, b.z0, owner);
            const int o_nx = __shfl_sync(0xffffffffu, b.nx, owner);
            const int o_ny = __shfl_sync(0xffffffffu, b.ny, owner);
            const int o_gid = __shfl_sync(0xffffffffu, gid, owner);
            if (k < total) {
                int r = k - o_excl;
                const int x = r % o_nx;
                r /= o_nx;
                const int y = r % o_ny;
                const int z = r / o_ny;
                const int tile =
                    ((o_z0 + z - tz0) * Ty + (o_y0 + y)) * Tx + (o_x0 + x);
                if (MODE == kCount) {
                    atomicAdd(counter + tile, 1);
                } else {
                    const int slot = atomicAdd(counter + tile, 1);
                    if (slot >= 0 && slot < capacity) {
                        ids_out[slot] = o_gid;
                    } else {
                        *error_flag = 1;
                    }
                }
            }
        }
    }
}

// ---- three-phase exclusive scan of per-tile counts ----------------------

__device__ __forceinline__ long long block_reduce_ll(long long v,
                                                     long long *smem) {
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if (lane == 0) smem[wid] = v;
    __syncthreads();
    long long t = 0;
    if (threadIdx.x < (blockDim.x >> 5)) t = smem[threadIdx.x];
    if (wid == 0) {
#pragma unroll
        for (int o = 16; o > 0; o >>= 1)
            t += __shfl_xor_sync(0xffffffffu, t, o);
    }
    __syncthreads();
    return t;  // valid in warp 0
}

// exclusive block scan of one value per thread; returns this thread's
// exclusive prefix and writes the block total to *total
__device__ __forceinline__ long long block_excl_scan_ll(long long v,
                                                        long long *smem,
                                                        long long *total) {
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    const int nw = blockDim.x >> 5;
    const long long incl = warp_inclusive_scan_ll(v);
    if (lane == 31) smem[wid] = incl;
    __syncthreads();
    if (wid == 0) {
        long long s = lane < nw ? smem[lane] : 0;
        s = warp_inclusive_scan_ll(s);
        if (lane < nw) smem[lane] = s;
    }
    __syncthreads();
    const long long warp_prefix = wid == 0 ? 0 : smem[wid - 1];
    *total = smem[nw - 1];
    __syncthreads();
    return warp_prefix + incl - v;
}

// ---- processing order by tile layer --------------------------------------
//
// With hundreds of millions of pairs the id array (4 B per pair) is far
// larger than L2, and the scatter's writes, random over that array, become
// DRAM read-modify-writes. Taking the Gaussians grouped by the (slab-
// relative) tile layer of their box's lower z corner keeps the warps in
// flight on a band of adjacent layers, whose segments stay in L2. The order
// is a counting sort of the Gaussians (not of the pairs) into one bucket
// per layer, plus a last bucket for Gaussians with no tile in the slab. Ids
// within a tile are sorted afterwards either way, so results do not change.

constexpr long long kOrderMinPairs = 1LL << 25;

__device__ __forceinline__ int layer_bucket(const int *tmin, const int *tmax,
                                            int i, int tz0, int tz1) {
    const Box b = load_box(tmin, tmax, i, tz0, tz1);
    return (b.nx > 0 && b.ny > 0 && b.nz > 0) ? b.z0 - tz0 : tz1 - tz0;
}

__global__ void __launch_bounds__(256)
layer_count_kernel(int n, const int *__restrict__ tmin,
                   const int *__restrict__ tmax, int tz0, int tz1,
                   int *__restrict__ counts) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    const unsigned active = __ballot_sync(0xffffffffu, i < n);
    if (i >= n) return;
    const int key = layer_bucket(tmin, tmax, i, tz0, tz1);
    const unsigned peers = __match_any_sync(active, key);
    if ((threadIdx.x & 31) == __ffs(peers) - 1)
        atomicAdd(&counts[key], __popc(peers));
}

// single CTA: counts -> exclusive offsets (the scatter's cursors), in place
__global__ void __launch_bounds__(1024)
layer_scan_kernel(int nb, int *__restrict__ counts) {
    __shared__ long long smem[32];
    const int per = (nb + 1023) / 1024;
    const int begin = threadIdx.x * per;
    long long local = 0;
    for (int k = 0; k < per; ++k)
        if (begin + k < nb) local += counts[begin + k];
    long long total;
    long long run = block_excl_scan_ll(local, smem, &total);
    for (int k = 0; k < per; ++k) {
        if (begin + k < nb) {
            const int v = counts[begin + k];
            counts[begin + k] = (int)run;
            run += v;
        }
    }
}

__global__ void __launch_bounds__(256)
layer_scatter_kernel(int n, const int *__restrict__ tmin,
                     const int *__restrict__ tmax, int tz0, int tz1,
                     int *__restrict__ cursor, int *__restrict__ order) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    const int lane = threadIdx.x & 31;
    const unsigned active = __ballot_sync(0xffffffffu, i < n);
    if (i >= n) return;
    const int key = layer_bucket(tmin, tmax, i, tz0, tz1);
    const unsigned peers = __match_any_sync(active, key);
    const int leader = __ffs(peers) - 1;
    int base = 0;
    if (lane == leader) base = atomicAdd(&cursor[key], __popc(peers));
    base = __shfl_sync(active, base, leader);
    order[base + __popc(peers & ((1u << lane) - 1u))] = i;
}

// Work items of the per-Gaussian backward for a tile of c pairs.
__device__ __forceinline__ int tile_items(int c) { return (c + 31) >> 5; }

// partials[b] = sum of block b's counts; with ipartials, ipartials[b] = sum
// of its work items (the backward's plan, scanned alongside the pairs)
__global__ void __launch_bounds__(kScanThreads)
scan_partials_kernel(const int *__restrict__ in, long long n,
                     long long *__restrict__ partials,
                     long long *__restrict__ ipartials) {
    __shared__ long long smem[32];
    const long long base = (long long)blockIdx.x * kScanTile;
    long long s = 0, si = 0;
#pragma unroll
    for (int k = 0; k < kScanItems; ++k) {
        const long long i = base + (long long)k * kScanThreads + threadIdx.x;
        if (i < n) {
            const int c = in[i];
            s += c;
            si += tile_items(c);
        }
    }
    s = block_reduce_ll(s, smem);
    if (threadIdx.x == 0) partials[blockIdx.x] = s;
    if (ipartials) {
        si = block_reduce_ll(si, smem);
        if (threadIdx.x == 0) ipartials[blockIdx.x] = si;
    }
}

// exclusive scan of p[0..nblocks) in place, grand total (clamped to
// total_cap) into p[nblocks]; returns the unclamped total
__device__ __forceinline__ long long scan_partials_block(long long *p,
                                                         int nblocks,
                                                         long long *smem,
                                                         long long total_cap) {
    const int per = (nblocks + 1023) / 1024;
    const int begin = threadIdx.x * per;
    long long local = 0;
    for (int k = 0; k < per; ++k)
        if (begin + k < nblocks) local += p[begin + k];
    long long total;
    long long run = block_excl_scan_ll(local, smem, &total);
    for (int k = 0; k < per; ++k) {
        if (begin + k < nblocks) {
            const long long v = p[begin + k];
            p[begin + k] = run;
            run += v;
        }
    }
    if (threadIdx.x == 0) p[nblocks] = min(total, total_cap);
    return total;
}

// single CTA: exclusive scans of the per-block partial sums (pairs, and
// items when given); the pair total also to count_out, with overflow_out =
// (total > cap). The item total is clamped to icap (the item buffer), as
// the item ranges are, so the backward never reads past the descriptors.
__global__ void __launch_bounds__(1024)
scan_partials_top_kernel(long long *__restrict__ partials,
                         long long *__restrict__ ipartials, int nblocks,
                         long long cap, long long icap,
                         long long *__restrict__ count_out,
                         float *__restrict__ overflow_out) {
    __shared__ long long smem[32];
    const long long total =
        scan_partials_block(partials, nblocks, smem, LLONG_MAX);
    if (threadIdx.x == 0) {
        if (count_out) *count_out = total;
        if (overflow_out) *overflow_out = total > cap ? 1.f : 0.f;
    }
    if (ipartials) {
        __syncthreads();
        scan_partials_block(ipartials, nblocks, smem, icap);
    }
}

// tile_bins[t] = count ? (offset, offset + count) : (0, 0); cursor[t] = offset.
// Offsets and ends are clamped to `cap` (the id buffer's capacity): when the
// pairs outnumber the buffer, every range still lies inside it, the scatter
// drops what does not fit, and the caller detects the overflow from the count.
// With ipartials, item_bins[t] = the tile's range of work items, clamped to
// icap (the item buffer) in the same way.
__global__ void __launch_bounds__(kScanThreads)
scan_bins_kernel(const int *__restrict__ counts, long long n,
                 const long long *__restrict__ partials,
                 int2 *__restrict__ tile_bins, int *__restrict__ cursor,
                 long long cap, const long long *__restrict__ ipartials,
                 int2 *__restrict__ item_bins, long long icap) {
    __shared__ long long smem[32];
    const long long base = (long long)blockIdx.x * kScanTile;
    // each thread owns kScanItems consecutive tiles
    const long long first = base + (long long)threadIdx.x * kScanItems;
    int v[kScanItems];
    long long s = 0, si = 0;
#pragma unroll
    for (int k = 0; k < kScanItems; ++k) {
        v[k] = (first + k < n) ? counts[first + k] : 0;
        s += v[k];
        si += tile_items(v[k]);
    }
    long long total;
    long long run = block_excl_scan_ll(s, smem, &total) + partials[blockIdx.x];
    long long irun = 0;
    if (ipartials)
        irun = block_excl_scan_ll(si, smem, &total) + ipartials[blockIdx.x];
#pragma unroll
    for (int k = 0; k < kScanItems; ++k) {
        if (first + k < n) {
            const int off = (int)min(run, cap);
            const int end = (int)min(run + v[k], cap);
            tile_bins[first + k] =
                v[k] > 0 ? make_int2(off, end) : make_int2(0, 0);
            cursor[first + k] = off;
            run += v[k];
            if (ipartials) {
                const int ni = tile_items(v[k]);
                item_bins[first + k] = make_int2((int)min(irun, icap),
                                                 (int)min(irun + ni, icap));
                irun += ni;
            }
        }
    }
}

// ---- per-tile segment sort ----------------------------------------------

// Bitonic sort of 32*K ints held K per lane (element e = k*32 + lane).
template <int K>
__device__ __forceinline__ void warp_bitonic(int (&v)[K], int lane) {
#pragma unroll
    for (int size = 2; size <= 32 * K; size <<= 1) {
#pragma unroll
        for (int stride = size >> 1; stride > 0; stride >>= 1) {
            if (stride >= 32) {
                const int ks = stride >> 5;
#pragma unroll
                for (int k = 0; k < K; ++k) {
                    if ((k & ks) == 0) {
                        const int e = k * 32 + lane;
                        const bool up = (e & size) == 0;
                        const int a = v[k], b = v[k | ks];
                        const int lo = min(a, b), hi = max(a, b);
                        v[k] = up ? lo : hi;
                        v[k | ks] = up ? hi : lo;
                    }
                }
            } else {
#pragma unroll
                for (int k = 0; k < K; ++k) {
                    const int e = k * 32 + lane;
                    const bool up = (e & size) == 0;
                    const int other = __shfl_xor_sync(0xffffffffu, v[k], stride);
                    const bool keep_min = ((e & stride) == 0) == up;
                    v[k] = keep_min ? min(v[k], other) : max(v[k], other);
                }
            }
        }
    }
}

template <int K>
__device__ __forceinline__ void warp_sort_segment(int *seg, int n, int lane) {
    int v[K];
#pragma unroll
    for (int k = 0; k < K; ++k) {
        const int e = k * 32 + lane;
        v[k] = e < n ? seg[e] : INT_MAX;
    }
    warp_bitonic<K>(v, lane);
#pragma unroll
    for (int k = 0; k < K; ++k) {
        const int e = k * 32 + lane;
        if (e < n) seg[e] = v[k];
    }
}

constexpr int kWarpSortMax = 256;
constexpr int kCtaSortMax = 16384;

// one warp per tile; large segments are queued for the CTA-level sorts
__global__ void __launch_bounds__(256)
sort_segments_warp_kernel(const int2 *__restrict__ tile_bins, long long ntiles,
                          int *__restrict__ ids, int *__restrict__ big_list,
                          int *__restrict__ big_count,
                          const int2 *__restrict__ item_bins,
                          int4 *__restrict__ item_desc) {
    const int lane = threadIdx.x & 31;
    const long long w0 = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const long long nw = ((long long)gridDim.x * blockDim.x) >> 5;
    for (long long t = w0; t < ntiles; t += nw) {
        const int2 r = tile_bins[t];
        if (item_desc) {
            // the backward's work items of this tile: (tile, first pair,
            // Gaussians <= 32)
            const int2 it = item_bins[t];
            for (int k = it.x + lane; k < it.y; k += 32) {
                const int start = r.x + 32 * (k - it.x);
                item_desc[k] =
                    make_int4((int)t, start, max(0, min(32, r.y - start)), 0);
            }
        }
        const int n = r.y - r.x;
        if (n <= 1) continue;
        int *seg = ids + r.x;
        if (n <= 32) warp_sort_segment<1>(seg, n, lane);
        else if (n <= 64) warp_sort_segment<2>(seg, n, lane);
        else if (n <= 128) warp_sort_segment<4>(seg, n, lane);
        else if (n <= kWarpSortMax) warp_sort_segment<8>(seg, n, lane);
        else if (lane == 0) big_list[atomicAdd(big_count, 1)] = (int)t;
    }
}

// one CTA per queued tile: bitonic sort in shared memory (n <= 16384), or a
// stable LSD radix sort on 4-bit digits through tmp (larger n)
__global__ void __launch_bounds__(1024)
sort_segments_cta_kernel(const int2 *__restrict__ tile_bins,
                         int *__restrict__ ids, int *__restrict__ tmp,
                         const int *__restrict__ big_list,
                         const int *__restrict__ big_count, int num_gaussians) {
    extern __shared__ int sm[];
    const int count = *big_count;
    for (int q = blockIdx.x; q < count; q += gridDim.x) {
        const int2 r = tile_bins[big_list[q]];
        const int n = r.y - r.x;
        int *seg = ids + r.x;
        if (n <= kCtaSortMax) {
            int P = 1;
            while (P < n) P <<= 1;
            for (int e = threadIdx.x; e < P; e += blockDim.x)
                sm[e] = e < n ? seg[e] : INT_MAX;
            __syncthreads();
            for (int size = 2; size <= P; size <<= 1) {
                for (int stride = size >> 1; stride > 0; stride >>= 1) {
                    for (int e = threadIdx.x; e < P / 2; e += blockDim.x) {
                        // pair (i, i + stride) with i having bit `stride` clear
                        const int i = 2 * e - (e & (stride - 1));
                        const int j = i + stride;
                        const bool up = (i & size) == 0;
                        const int a = sm[i], b = sm[j];
                        if ((a > b) == up) {
                            sm[i] = b;
                            sm[j] = a;
                        }
                    }
                    __syncthreads();
                }
            }
            for (int e = threadIdx.x; e < n; e += blockDim.x) seg[e] = sm[e];
            __syncthreads();
        } else {
            // stable LSD radix sort, 4 bits per pass, chunks of blockDim.x
            int bits = 1;
            while ((1 << bits) < num_gaussians && bits < 31) ++bits;
            int *src = seg, *dst = tmp + r.x;
            int *hist = sm;           // 16 digit counters
            int *warp_cnt = sm + 16;  // [32 warps][16 digits]
            const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
            const int nwarps = blockDim.x >> 5;
            for (int shift = 0; shift < bits; shift += 4) {
                if (threadIdx.x < 16) hist[threadIdx.x] = 0;
                __syncthreads();
                for (int e = threadIdx.x; e < n; e += blockDim.x)
                    atomicAdd(&hist[(src[e] >> shift) & 15], 1);
                __syncthreads();
                if (threadIdx.x == 0) {
                    int run = 0;
                    for (int d = 0; d < 16; ++d) {
                        const int c = hist[d];
                        hist[d] = run;
                        run += c;
                    }
                }
                __syncthreads();
                for (int base = 0; base < n; base += blockDim.x) {
                    const int e = base + threadIdx.x;
                    const bool valid = e < n;
                    const int key = valid ? src[e] : 0;
                    const int dig = valid ? ((key >> shift) & 15) : 16;
                    unsigned my_mask = 0, my_rank = 0;
#pragma unroll
                    for (int d = 0; d < 16; ++d) {
                        const unsigned m = __ballot_sync(0xffffffffu, dig == d);
                        if (lane == 0) warp_cnt[wid * 16 + d] = __popc(m);
                        if (dig == d) {
                            my_mask = m;
                            my_rank = __popc(m & ((1u << lane) - 1));
                        }
                    }
                    (void)my_mask;
                    __syncthreads();
                    if (valid) {
                        int before = 0;
                        for (int w = 0; w < wid; ++w)
                            before += warp_cnt[w * 16 + dig];
                        dst[hist[dig] + before + (int)my_rank] = key;
                    }
                    __syncthreads();
                    if (threadIdx.x < 16) {
                        int add = 0;
                        for (int w = 0; w < nwarps; ++w)
                            add += warp_cnt[w * 16 + threadIdx.x];
                        hist[threadIdx.x] += add;
                    }
                    __syncthreads();
                }
                int *t = src;
                src = dst;
                dst = t;
                __syncthreads();
            }
            if (src != seg) {
                for (int e = threadIdx.x; e < n; e += blockDim.x)
                    seg[e] = src[e];
            }
            __syncthreads();
        }
    }
}

}  // namespace

// Workspace layout (all 256-byte aligned):
//   counts  [T]  int  (reused as scatter cursors)
//   partials[nblocks+1] long long
//   big_list[T]  int, big_count int, error flag int
//   tmp     [I]  int  (radix temporary for huge segments)
struct BinLayout {
    size_t counts, partials, big_list, flags, tmp, layer, order, total;
    bool ordered;  // Gaussians taken in tile-layer order (large pair counts)
};

static inline size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

static bool use_layer_order(long long nisect, long long layers) {
    return nisect >= kOrderMinPairs && layers > 1;
}

BinLayout bin_layout(long long ntiles, long long nisect, long long n,
                     long long layers) {
    BinLayout L;
    const long long nblocks = (ntiles + kScanTile - 1) / kScanTile;
    size_t off = 0;
    L.counts = off;
    off = align256(off + sizeof(int) * (size_t)ntiles);
    L.partials = off;
    off = align256(off + sizeof(long long) * (size_t)(nblocks + 1));
    L.big_list = off;
    off = align256(off + sizeof(int) * (size_t)ntiles);
    L.flags = off;
    off = align256(off + sizeof(int) * 4);
    L.tmp = off;
    off = align256(off + sizeof(int) * (size_t)nisect);
    L.ordered = use_layer_order(nisect, layers);
    L.layer = off;
    if (L.ordered) off = align256(off + sizeof(int) * (size_t)(layers + 1));
    L.order = off;
    if (L.ordered) off = align256(off + sizeof(int) * (size_t)(n > 0 ? n : 1));
    L.total = off;
    return L;
}

size_t bin_workspace_bytes(long long ntiles, long long nisect, long long n,
                           long long layers) {
    return bin_layout(ntiles, nisect, n, layers).total;
}

// The pair total that the binning's scan left in its workspace.
const long long *bin_pair_total(const void *ws, long long ntiles) {
    const BinLayout L = bin_layout(ntiles, 0, 0, 1);
    return reinterpret_cast<const long long *>(
               static_cast<const char *>(ws) + L.partials) +
           scan_blocks(ntiles);
}

long long scan_blocks(long long ntiles) {
    return (ntiles + kScanTile - 1) / kScanTile;
}

// Exclusive scan of per-tile counts into tile_bins / cursors (counts is
// overwritten with the cursors), ranges clamped to `cap`; the grand total is
// left in partials[scan_blocks(ntiles)] and, when given, in count_out, with
// overflow_out = (total > cap). With `items` the backward's work items per
// tile are scanned too (see ItemScan). Exposed for the backward planner.
cudaError_t scan_counts_to_bins(int *counts, long long ntiles,
                                long long *partials, int *tile_bins,
                                cudaStream_t stream, long long cap,
                                long long *count_out, float *overflow_out,
                                const ItemScan *items) {
    const long long nblocks = scan_blocks(ntiles);
    if (nblocks > 1024LL * 64) return cudaErrorInvalidValue;
    long long *ip = items ? items->partials : nullptr;
    scan_partials_kernel<<<(unsigned)nblocks, kScanThreads, 0, stream>>>(
        counts, ntiles, partials, ip);
    scan_partials_top_kernel<<<1, 1024, 0, stream>>>(
        partials, ip, (int)nblocks, cap, items ? items->cap : 0, count_out,
        overflow_out);
    scan_bins_kernel<<<(unsigned)nblocks, kScanThreads, 0, stream>>>(
        counts, ntiles, partials, reinterpret_cast<int2 *>(tile_bins), counts,
        cap, ip, items ? reinterpret_cast<int2 *>(items->item_bins) : nullptr,
        items ? items->cap : 0);
    count_launches(3);
    return cudaGetLastError();
}

cudaError_t launch_binning(int n, long long nisect, const int *tmin,
                           const int *tmax, int Tx, int Ty, int tz0, int tz1,
                           int *ids_out, int *tile_bins, void *ws,
                           cudaStream_t stream, long long *count_out,
                           float *overflow_out, const ItemScan *items) {
    const long long ntiles = (long long)(tz1 - tz0) * Ty * Tx;
    const BinLayout L = bin_layout(ntiles, nisect, n, tz1 - tz0);
    char *base = static_cast<char *>(ws);
    int *counts = reinterpret_cast<int *>(base + L.counts);
    long long *partials = reinterpret_cast<long long *>(base + L.partials);
    int *big_list = reinterpret_cast<int *>(base + L.big_list);
    int *flags = reinterpret_cast<int *>(base + L.flags);
    int *tmp = reinterpret_cast<int *>(base + L.tmp);

    cudaError_t err;
    if ((err = cudaMemsetAsync(counts, 0, sizeof(int) * ntiles, stream)))
        return err;
    if ((err = cudaMemsetAsync(flags, 0, sizeof(int) * 4, stream))) return err;
    if (ntiles == 0) {
        if (count_out &&
            (err = cudaMemsetAsync(count_out, 0, sizeof(long long), stream)))
            return err;
        if (overflow_out &&
            (err = cudaMemsetAsync(overflow_out, 0, sizeof(float), stream)))
            return err;
        return cudaSuccess;
    }
    const int *order = nullptr;
    if (L.ordered && n > 0 && nisect > 0) {
        int *layer = reinterpret_cast<int *>(base + L.layer);
        int *ord = reinterpret_cast<int *>(base + L.order);
        const int nb = tz1 - tz0 + 1;
        if ((err = cudaMemsetAsync(layer, 0, sizeof(int) * nb, stream)))
            return err;
        const unsigned gb = (unsigned)((n + 255) / 256);
        layer_count_kernel<<<gb, 256, 0, stream>>>(n, tmin, tmax, tz0, tz1,
                                                   layer);
        layer_scan_kernel<<<1, 1024, 0, stream>>>(nb, layer);
        layer_scatter_kernel<<<gb, 256, 0, stream>>>(n, tmin, tmax, tz0, tz1,
                                                     layer, ord);
        count_launches(3);
        order = ord;
    }
    if (n > 0 && (nisect > 0 || count_out || overflow_out)) {
        const int warps = (n + 31) / 32;
        const int blocks = min((warps + 7) / 8, kSMs * 16);
        expand_pairs_kernel<kCount><<<blocks, 256, 0, stream>>>(
            n, tmin, tmax, Tx, Ty, tz0, tz1, counts, nullptr, 0, flags + 1,
            order);
        count_launches(1);
    }
    if ((err = scan_counts_to_bins(counts, ntiles, partials, tile_bins, stream,
                                   nisect, count_out, overflow_out, items)))
        return err;
    if (n <= 0 || nisect <= 0) return cudaGetLastError();
    {
        const int warps = (n + 31) / 32;
        const int blocks = min((warps + 7) / 8, kSMs * 16);
        expand_pairs_kernel<kScatter><<<blocks, 256, 0, stream>>>(
            n, tmin, tmax, Tx, Ty, tz0, tz1, counts, ids_out, nisect,
            flags + 1, order);
    }
    {
        const long long warps_needed = ntiles;
        const long long blocks =
            std::min<long long>((warps_needed + 7) / 8, (long long)kSMs * 32);
        sort_segments_warp_kernel<<<(unsigned)blocks, 256, 0, stream>>>(
            reinterpret_cast<const int2 *>(tile_bins), ntiles, ids_out,
            big_list, flags,
            items ? reinterpret_cast<const int2 *>(items->item_bins) : nullptr,
            items ? items->desc : nullptr);
    }
    sort_segments_cta_kernel<<<kSMs * 2, 1024, kCtaSortMax * sizeof(int),
                               stream>>>(
        reinterpret_cast<const int2 *>(tile_bins), ids_out, tmp, big_list,
        flags, n);
    count_launches(3);
    return cudaGetLastError();
}

// The CTA-level segment sort keeps up to kCtaSortMax ids in shared memory;
// opt in to that much dynamic shared memory once per device.
void enable_large_smem() {
    static int done_mask = 0;
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 32 && (done_mask >> dev) & 1) return;
    cudaFuncSetAttribute(sort_segments_cta_kernel,
                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                         kCtaSortMax * (int)sizeof(int));
    if (dev < 32) done_mask |= 1 << dev;
}

// Number of (tile, gaussian) pairs with tile z in [tz0, tz1).
__global__ void __launch_bounds__(256)
count_slab_pairs_kernel(int n, const int *__restrict__ tmin,
                        const int *__restrict__ tmax, int tz0, int tz1,
                        unsigned long long *__restrict__ out) {
    __shared__ long long smem[32];
    long long s = 0;
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n;
         i += (long long)gridDim.x * blockDim.x) {
        const Box b = load_box(tmin, tmax, (int)i, tz0, tz1);
        s += (long long)b.nx * b.ny * b.nz;
    }
    s = block_reduce_ll(s, smem);
    if (threadIdx.x == 0 && s) atomicAdd(out, (unsigned long long)s);
}

cudaError_t launch_count_slab_pairs(int n, const int *tmin, const int *tmax,
                                    int tz0, int tz1, long long *out,
                                    cudaStream_t stream) {
    cudaError_t err = cudaMemsetAsync(out, 0, sizeof(long long), stream);
    if (err) return err;
    if (n <= 0) return cudaSuccess;
    const int blocks = std::min((n + 255) / 256, kSMs * 8);
    count_slab_pairs_kernel<<<blocks, 256, 0, stream>>>(
        n, tmin, tmax, tz0, tz1, reinterpret_cast<unsigned long long *>(out));
    count_launches(1);
    return cudaGetLastError();
}

}  // namespace gsv
