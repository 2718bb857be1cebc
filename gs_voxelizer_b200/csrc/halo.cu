// Halo exchange for owner-sharded Gaussians (z-slab sharding, one process
// per GPU). Not part of the reference, which is single-GPU.
//
// Every rank owns a subset of the Gaussians (normally those whose centre
// lies in its slab) and projects only those. An owned Gaussian whose tile
// box reaches another rank's slab is sent there as a render record; each
// rank voxelizes its slab with its owned Gaussians plus the records it
// received (its halo), and sends the halo's gradients back to their owners,
// which add them up in rank order. Traffic and per-rank work scale with the
// halo, not with the number of ranks.
//
// Buffers hold one segment per peer rank: a header record followed by `cap`
// record slots. Slots are assigned by a prefix scan over the owner's
// Gaussian index, so the order of a halo (and with it every result) is
// deterministic.
#include "common.cuh"

namespace gsv {

constexpr int kHaloScan = 1024;

namespace {

__device__ __forceinline__ bool box_meets_slab(const int *tmin, const int *tmax,
                                               int i, int tz0, int tz1) {
    const int x0 = tmin[3 * i + 0], y0 = tmin[3 * i + 1], z0 = tmin[3 * i + 2];
    const int x1 = tmax[3 * i + 0], y1 = tmax[3 * i + 1], z1 = tmax[3 * i + 2];
    return x1 > x0 && y1 > y0 && min(z1, tz1) > max(z0, tz0);
}

// counts[b * world + d] = owned Gaussians of block b sent to rank d
__global__ void __launch_bounds__(kHaloScan)
halo_count_kernel(int n, const int *__restrict__ tmin,
                  const int *__restrict__ tmax, HaloPeers P,
                  int *__restrict__ counts) {
    __shared__ int sc[kHaloMaxRanks];
    for (int d = threadIdx.x; d < P.world; d += blockDim.x) sc[d] = 0;
    __syncthreads();
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    for (int d = 0; d < P.world; ++d) {
        const bool send = d != P.rank && i < n &&
                          box_meets_slab(tmin, tmax, i, P.tz0[d], P.tz1[d]);
        const unsigned m = __ballot_sync(0xffffffffu, send);
        if ((threadIdx.x & 31) == 0 && m) atomicAdd(&sc[d], __popc(m));
    }
    __syncthreads();
    for (int d = threadIdx.x; d < P.world; d += blockDim.x)
        counts[blockIdx.x * P.world + d] = sc[d];
}

// single CTA: exclusive scan of the block counts per destination, totals
// into totals[d]
__global__ void __launch_bounds__(kHaloMaxRanks)
halo_scan_kernel(int nblocks, HaloPeers P, int *__restrict__ counts,
                 long long *__restrict__ totals) {
    const int d = threadIdx.x;
    if (d >= P.world) return;
    long long run = 0;
    for (int b = 0; b < nblocks; ++b) {
        const int c = counts[b * P.world + d];
        counts[b * P.world + d] = (int)run;
        run += c;
    }
    totals[d] = run;
}

// Writes each sent Gaussian's record into its destination's segment at the
// slot given by the scan (slots past the capacity are dropped and flagged),
// and slot_map[i * world + d] = slot or -1.
__global__ void __launch_bounds__(kHaloScan)
halo_pack_kernel(int n, int C, const float4 *__restrict__ pr,
                 const float2 *__restrict__ cq, const float *__restrict__ inten,
                 const int *__restrict__ tmin, const int *__restrict__ tmax,
                 HaloPeers P, const int *__restrict__ block_base,
                 int *__restrict__ slot_map) {
    __shared__ int warp_base[kHaloScan / 32];
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    for (int d = 0; d < P.world; ++d) {
        if (d == P.rank) {
            if (i < n) slot_map[(size_t)i * P.world + d] = -1;
            continue;
        }
        const bool send_it =
            i < n && box_meets_slab(tmin, tmax, i, P.tz0[d], P.tz1[d]);
        const unsigned m = __ballot_sync(0xffffffffu, send_it);
        __syncthreads();
        if (lane == 0) warp_base[wid] = __popc(m);
        __syncthreads();
        if (threadIdx.x == 0) {  // exclusive scan of the warp counts
            int run = 0;
            for (int w = 0; w < (int)(blockDim.x >> 5); ++w) {
                const int c = warp_base[w];
                warp_base[w] = run;
                run += c;
            }
        }
        __syncthreads();
        if (i < n) {
            int slot = -1;
            if (send_it) {
                const int s = block_base[blockIdx.x * P.world + d] +
                              warp_base[wid] + __popc(m & ((1u << lane) - 1u));
                if (s < P.cap[d]) {
                    slot = s;
                    float *r = P.dst[d] + (1 + s) * kHaloRec;
                    const float4 p = pr[i];
                    reinterpret_cast<float4 *>(r)[0] = p;
                    const float2 a = cq[3 * i], b = cq[3 * i + 1], c = cq[3 * i + 2];
                    reinterpret_cast<float4 *>(r)[1] = make_float4(a.x, a.y, b.x, b.y);
                    float I[4] = {0.f, 0.f, 0.f, 0.f};
                    for (int k = 0; k < C; ++k) I[k] = inten[(size_t)i * C + k];
                    reinterpret_cast<float4 *>(r)[2] = make_float4(c.x, c.y, I[0], I[1]);
                    reinterpret_cast<float4 *>(r)[3] = make_float4(
                        I[2], I[3], __int_as_float(tmin[3 * i]),
                        __int_as_float(tmin[3 * i + 1]));
                    reinterpret_cast<float4 *>(r)[4] = make_float4(
                        __int_as_float(tmin[3 * i + 2]), __int_as_float(tmax[3 * i]),
                        __int_as_float(tmax[3 * i + 1]),
                        __int_as_float(tmax[3 * i + 2]));
                }
            }
            slot_map[(size_t)i * P.world + d] = slot;
        }
    }
}

// Header record of each destination segment: [count (int bits), overflow];
// counts_out[d] (optional) = unclamped number of Gaussians for rank d
__global__ void halo_header_kernel(HaloPeers P, const long long *__restrict__ totals,
                                   long long *__restrict__ counts_out) {
    const int d = threadIdx.x;
    if (d >= P.world) return;
    if (counts_out) counts_out[d] = d == P.rank ? 0 : totals[d];
    if (d == P.rank) return;
    float *h = P.dst[d];
    const long long t = totals[d];
    h[0] = __int_as_float((int)(t < P.cap[d] ? t : (long long)P.cap[d]));
    h[1] = t > P.cap[d] ? 1.f : 0.f;
}

// Received records -> local arrays at index n_own + loff[s] + slot; unused
// slots become Gaussians with an empty tile box (no pairs).
__global__ void __launch_bounds__(256)
halo_unpack_kernel(int n_own, int C, HaloPeers R, long long total_slots,
                   const float *__restrict__ recv,
                   float4 *__restrict__ pr, float2 *__restrict__ cq,
                   float *__restrict__ inten, int *__restrict__ tmin,
                   int *__restrict__ tmax, float *__restrict__ flags) {
    const long long g = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    // Every peer's segment starts with its header, also when this rank gave
    // it no slots: thread k reads peer k's overflow bit, so a sender that
    // had Gaussians for a zero-capacity segment is still detected.
    if (g < R.world && g != R.rank && recv[R.off[g] * kHaloRec + 1] != 0.f)
        flags[1] = 1.f;
    if (g >= total_slots) return;
    // source of this slot
    int s = 0;
    for (int k = 0; k < R.world; ++k)
        if (k != R.rank && R.cap[k] > 0 && g >= R.loff[k]) s = k;
    const int slot = (int)(g - R.loff[s]);
    const float *h = recv + R.off[s] * kHaloRec;
    const int count = __float_as_int(h[0]);
    const long long li = n_own + g;
    if (slot < count) {
        const float *r = recv + (R.off[s] + 1 + slot) * kHaloRec;
        const float4 a = reinterpret_cast<const float4 *>(r)[0];
        const float4 b = reinterpret_cast<const float4 *>(r)[1];
        const float4 c = reinterpret_cast<const float4 *>(r)[2];
        const float4 d = reinterpret_cast<const float4 *>(r)[3];
        const float4 e = reinterpret_cast<const float4 *>(r)[4];
        pr[li] = a;
        cq[3 * li] = make_float2(b.x, b.y);
        cq[3 * li + 1] = make_float2(b.z, b.w);
        cq[3 * li + 2] = make_float2(c.x, c.y);
        const float I[4] = {c.z, c.w, d.x, d.y};
        for (int k = 0; k < C; ++k) inten[li * C + k] = I[k];
        tmin[3 * li] = __float_as_int(d.z);
        tmin[3 * li + 1] = __float_as_int(d.w);
        tmin[3 * li + 2] = __float_as_int(e.x);
        tmax[3 * li] = __float_as_int(e.y);
        tmax[3 * li + 1] = __float_as_int(e.z);
        tmax[3 * li + 2] = __float_as_int(e.w);
    } else {
        pr[li] = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int k = 0; k < 3; ++k) cq[3 * li + k] = make_float2(0.f, 0.f);
        for (int k = 0; k < C; ++k) inten[li * C + k] = 0.f;
        for (int k = 0; k < 3; ++k) {
            tmin[3 * li + k] = 0;
            tmax[3 * li + k] = 0;
        }
    }
}

// Gradients of the halo entries -> their owners' segments (same slots);
// header [loss, overflow] of this rank in every segment.
__global__ void __launch_bounds__(256)
halo_pack_grads_kernel(int n_own, int C, HaloPeers R, long long total_slots,
                       const float4 *__restrict__ gp,
                       const float2 *__restrict__ gc, const float *__restrict__ gi,
                       const float *__restrict__ loss, const float *__restrict__ flags) {
    const long long g = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (g < R.world && g != R.rank) {
        float *h = R.dst[g];
        h[0] = loss[0];
        h[1] = fmaxf(flags[0], flags[1]);
    }
    if (g >= total_slots) return;
    int s = 0;
    for (int k = 0; k < R.world; ++k)
        if (k != R.rank && R.cap[k] > 0 && g >= R.loff[k]) s = k;
    const int slot = (int)(g - R.loff[s]);
    const long long li = n_own + g;
    float *r = R.dst[s] + (1 + slot) * kHaloGrad;
    reinterpret_cast<float4 *>(r)[0] = gp[li];
    const float2 a = gc[3 * li], b = gc[3 * li + 1], c = gc[3 * li + 2];
    reinterpret_cast<float4 *>(r)[1] = make_float4(a.x, a.y, b.x, b.y);
    float I[4] = {0.f, 0.f, 0.f, 0.f};
    for (int k = 0; k < C; ++k) I[k] = gi[li * C + k];
    reinterpret_cast<float4 *>(r)[2] = make_float4(c.x, c.y, I[0], I[1]);
    reinterpret_cast<float4 *>(r)[3] = make_float4(I[2], I[3], 0.f, 0.f);
}

// Owner side: add the peers' gradients for each owned Gaussian in rank
// order (deterministic); thread 0 also sums the ranks' losses in rank order
// and ORs their overflow flags into out[0..1].
__global__ void __launch_bounds__(256)
halo_accumulate_kernel(int n, int C, HaloPeers P, const int *__restrict__ slot_map,
                       const float *__restrict__ recv, float4 *__restrict__ gp,
                       float2 *__restrict__ gc, float *__restrict__ gi,
                       const float *__restrict__ loss, const float *__restrict__ flags,
                       float *__restrict__ out) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i == 0) {
        float l = 0.f, f = 0.f;
        for (int d = 0; d < P.world; ++d) {
            if (d == P.rank) {
                l += loss[0];
                f = fmaxf(f, fmaxf(flags[0], flags[1]));
            } else {
                const float *h = recv + P.off[d] * kHaloGrad;
                l += h[0];
                f = fmaxf(f, h[1]);
            }
        }
        out[0] = l;
        out[1] = f;
    }
    if (i >= n) return;
    float4 p = gp[i];
    float2 a = gc[3 * i], b = gc[3 * i + 1], c = gc[3 * i + 2];
    float I[4] = {0.f, 0.f, 0.f, 0.f};
    for (int k = 0; k < C; ++k) I[k] = gi[(size_t)i * C + k];
    bool any = false;
    for (int d = 0; d < P.world; ++d) {
        const int slot = slot_map[(size_t)i * P.world + d];
        if (slot < 0) continue;
        any = true;
        const float *r = recv + (P.off[d] + 1 + slot) * kHaloGrad;
        const float4 q0 = reinterpret_cast<const float4 *>(r)[0];
        const float4 q1 = reinterpret_cast<const float4 *>(r)[1];
        const float4 q2 = reinterpret_cast<const float4 *>(r)[2];
        const float4 q3 = reinterpret_cast<const float4 *>(r)[3];
        p.x += q0.x; p.y += q0.y; p.z += q0.z; p.w += q0.w;
        a.x += q1.x; a.y += q1.y; b.x += q1.z; b.y += q1.w;
        c.x += q2.x; c.y += q2.y;
        I[0] += q2.z; I[1] += q2.w; I[2] += q3.x; I[3] += q3.y;
    }
    if (!any) return;
    gp[i] = p;
    gc[3 * i] = a;
    gc[3 * i + 1] = b;
    gc[3 * i + 2] = c;
    for (int k = 0; k < C; ++k) gi[(size_t)i * C + k] = I[k];
}

// Device barrier across the ranks' GPUs, for the direct-write exchange.
// Every rank holds a signal array of `world` ints in memory its peers can
// write (symmetric memory over NVLink); sig[d] is rank d's device address of
// its array. A call takes the next epoch from the rank's own counter, stores
// it (release, system scope) into slot `rank` of every peer's array, and
// waits until every peer's slot in its own array has reached it (acquire
// loads). Epochs only grow, so the barrier needs no reset and can be
// replayed inside a CUDA graph. The kernels before it on the stream (the
// packing kernels' stores into the peers' buffers) have completed when it
// starts; the release store orders them before the signal. Each wait is
// bounded: on timeout the kernel records an error in g_peer_error and
// returns.
__device__ int g_peer_error = 0;

struct PeerSig {
    int *sig[kHaloMaxRanks];
};

constexpr long long kPeerSpinLimit = 1LL << 22;  // polls of ~0.5 us

__global__ void __launch_bounds__(kHaloMaxRanks)
peer_barrier_kernel(int world, int rank, PeerSig S, int *__restrict__ epoch) {
    __shared__ int e;
    if (threadIdx.x == 0) {
        e = *epoch + 1;
        *epoch = e;
    }
    __syncthreads();
    const int d = threadIdx.x;
    if (d < world && d != rank) {
        __threadfence_system();
        asm volatile("st.release.sys.global.s32 [%0], %1;" ::"l"(S.sig[d] + rank),
                     "r"(e)
                     : "memory");
        const int *mine = S.sig[rank] + d;
        int v = 0;
        for (long long it = 0; it < kPeerSpinLimit; ++it) {
            asm volatile("ld.acquire.sys.global.s32 %0, [%1];" : "=r"(v) : "l"(mine)
                         : "memory");
            if (v >= e) break;
            __nanosleep(500);
        }
        if (v < e) atomicExch(&g_peer_error, 1);
    }
    __syncthreads();
    __threadfence_system();
}

}  // namespace

cudaError_t launch_peer_barrier(int world, int rank, const long long *sig_ptrs,
                                int *epoch, cudaStream_t stream) {
    PeerSig S;
    for (int d = 0; d < kHaloMaxRanks; ++d)
        S.sig[d] = d < world ? reinterpret_cast<int *>(
                                   static_cast<uintptr_t>(sig_ptrs[d]))
                             : nullptr;
    peer_barrier_kernel<<<1, kHaloMaxRanks, 0, stream>>>(world, rank, S, epoch);
    count_launches(1);
    return cudaGetLastError();
}

int peer_error_flag(bool clear) {
    int v = 0;
    if (cudaMemcpyFromSymbol(&v, g_peer_error, sizeof(int)) != cudaSuccess) return -1;
    if (clear && v) {
        const int zero = 0;
        if (cudaMemcpyToSymbol(g_peer_error, &zero, sizeof(int)) != cudaSuccess)
            return -1;
    }
    return v;
}

size_t halo_workspace_bytes(int n, int world) {
    const size_t nb = (size_t)((n + kHaloScan - 1) / kHaloScan);
    return ((nb * world * sizeof(int) + 255) & ~size_t(255)) +
           ((world * sizeof(long long) + 255) & ~size_t(255));
}

cudaError_t launch_halo_pack(int n, int C, const float *pr, const float *cq,
                             const float *inten, const int *tmin,
                             const int *tmax, const HaloPeers &P,
                             int *slot_map, long long *counts_out, void *ws,
                             cudaStream_t stream) {
    const int nb = (n + kHaloScan - 1) / kHaloScan;
    int *counts = static_cast<int *>(ws);
    long long *totals = reinterpret_cast<long long *>(
        static_cast<char *>(ws) +
        (((size_t)nb * P.world * sizeof(int) + 255) & ~size_t(255)));
    if (nb > 0) {
        halo_count_kernel<<<nb, kHaloScan, 0, stream>>>(n, tmin, tmax, P, counts);
        count_launches(1);
    }
    halo_scan_kernel<<<1, kHaloMaxRanks, 0, stream>>>(nb, P, counts, totals);
    if (nb > 0)
        halo_pack_kernel<<<nb, kHaloScan, 0, stream>>>(
            n, C, reinterpret_cast<const float4 *>(pr),
            reinterpret_cast<const float2 *>(cq), inten, tmin, tmax, P, counts,
            slot_map);
    halo_header_kernel<<<1, kHaloMaxRanks, 0, stream>>>(P, totals, counts_out);
    count_launches(nb > 0 ? 3 : 2);
    return cudaGetLastError();
}

cudaError_t launch_halo_unpack(int n_own, int C, const HaloPeers &R,
                               long long total_slots, const float *recv,
                               float *pr, float *cq, float *inten, int *tmin,
                               int *tmax, float *flags, cudaStream_t stream) {
    const long long threads = std::max<long long>(total_slots, R.world);
    const unsigned blocks = (unsigned)((threads + 255) / 256);
    halo_unpack_kernel<<<blocks, 256, 0, stream>>>(
        n_own, C, R, total_slots, recv, reinterpret_cast<float4 *>(pr),
        reinterpret_cast<float2 *>(cq), inten, tmin, tmax, flags);
    count_launches(1);
    return cudaGetLastError();
}

cudaError_t launch_halo_pack_grads(int n_own, int C, const HaloPeers &R,
                                   long long total_slots, const float *gp,
                                   const float *gc, const float *gi,
                                   const float *loss, const float *flags,
                                   cudaStream_t stream) {
    const long long threads = std::max<long long>(total_slots, R.world);
    const unsigned blocks = (unsigned)((threads + 255) / 256);
    halo_pack_grads_kernel<<<blocks, 256, 0, stream>>>(
        n_own, C, R, total_slots, reinterpret_cast<const float4 *>(gp),
        reinterpret_cast<const float2 *>(gc), gi, loss, flags);
    count_launches(1);
    return cudaGetLastError();
}

cudaError_t launch_halo_accumulate(int n, int C, const HaloPeers &P,
                                   const int *slot_map, const float *recv,
                                   float *gp, float *gc, float *gi,
                                   const float *loss, const float *flags,
                                   float *out, cudaStream_t stream) {
    const unsigned blocks = (unsigned)((std::max(n, 1) + 255) / 256);
    halo_accumulate_kernel<<<blocks, 256, 0, stream>>>(
        n, C, P, slot_map, recv, reinterpret_cast<float4 *>(gp),
        reinterpret_cast<float2 *>(gc), gi, loss, flags, out);
    count_launches(1);
    return cudaGetLastError();
}

}  // namespace gsv

