// Per-Gaussian backward of the fused-L1 voxelization on the 5th-generation
// tensor cores (tcgen05 + tensor memory), one channel.
//
// Semantics: gs_voxelizer/cuda/voxelize.cu:368-574 of the reference (the
// per-Gaussian backward), with dL/dvol = sign(vol - target) * grad_loss /
// denom (the fused L1 loss). For every (tile, Gaussian) pair the gradient
// needs ten weighted sums over the tile's voxels v,
//     S_k = sum_v alpha(v) g(v) phi_k(v),
//     phi = (1, qx, qy, qz, qx^2, qy^2, -, qx qy, qx qz, qy qz),
// with alpha = exp(sigma) culled as the reference culls it, g = sign of the
// loss gradient and q the voxel centre in half-voxel units. That is a matrix
// product A * B with A[row, v] = alpha g (a row per (pair, z-quarter of the
// tile)) and a constant B[v, k] = phi_k(v): the CUDA cores evaluate A and
// the tensor cores accumulate it.
//
// Layout of the work: a pack is 32 consecutive (tile, Gaussian) pairs of the
// tile-sorted pair list; its 128 rows are (quarter u = producer warp, pair =
// lane), each row covering the 128 voxels of one z-quarter (2 z-layers) of
// its pair's tile. Per 32-voxel chunk a producer lane evaluates its row,
// splits alpha * g into a tf32 high part and the remainder (together ~22
// significant bits, so the products keep float32 accuracy), and stores both
// into tensor memory; one thread of the CTA's MMA warp then issues
//     D[128 x 16] += [A_hi | A_lo] (TMEM, 128 x 64) * [B_c ; B_c] (smem, 64 x 16)
// as eight kind::tf32 MMAs (K = 8 each). The 16 D columns of a row hold its
// moments; the producers read them back (tcgen05.ld), convert them to the
// sums about the Gaussian centre, add the four quarters and issue the
// per-Gaussian atomics.
//
// g comes from a per-tile sign plane (tile-major, 512 floats per tile,
// +-2^64 or 0) that the fused forward writes in its epilogue, and the tile of
// every pair from a tile_of array written by the forward as well. The factor
// 2^64 keeps alpha' g (alpha' = 2^(sigma log2 e - thr - 126), flushed to 0
// below the cull threshold exactly as in the CUDA-core kernel) far from the
// float32 subnormal range, so the tf32 split loses nothing.
//
// Pipelining: two A buffers in tensor memory (chunk n+1 is evaluated while
// the MMAs of chunk n run), mbarriers between the producer warps and the MMA
// warp (full: chunk stored; empty: its MMAs completed; dfull: the pack's
// moments are ready). Every wait is bounded; on timeout the kernel records
// an error in g_tc_error, skips the remaining work and still releases its
// tensor memory.
#include "common.cuh"

namespace gsv {

// Nonzero after a tensor-core backward gave up on a barrier wait (no
// result of that launch can be trusted); read and cleared through the C ABI.
__device__ int g_tc_error = 0;

namespace {

constexpr int kTcProducerWarps = 4;
constexpr int kTcThreads = (kTcProducerWarps + 1) * 32;  // + MMA warp
constexpr int kTcPairs = 32;        // pairs per pack (lanes)
constexpr int kTcChunk = 32;        // voxels per K chunk
constexpr int kTcChunks = 4;        // chunks per z-quarter (128 voxels)
constexpr int kTcCols = 256;        // tensor-memory columns per CTA
constexpr int kTcBufs = 3;          // A buffers (chunks in flight)
constexpr int kTcBufCols = 2 * kTcChunk;  // A buffer: hi | lo
constexpr int kTcDCol = kTcBufs * kTcBufCols;  // D after the A buffers
constexpr int kTcN = 16;            // D columns (10 moments + padding)
constexpr int kTcSums = 10;
constexpr float kLn2 = 0.6931471805599453f;
constexpr int kTcRedStride = kTcSums + 1;  // smem row stride (bank spread)
// one B slab per MMA: N = 16 rows x K = 8 tf32 = 4 core matrices of
// 8 rows x 16 bytes; core matrices K-adjacent 128 B apart (LBO), N-adjacent
// 256 B apart (SBO)
constexpr int kTcSlabBytes = 512;
constexpr int kTcBBytes = kTcChunks * (2 * kTcChunk / 8) * kTcSlabBytes;  // 16 KB
// dynamic shared memory requested so that at most two CTAs share an SM
// (each allocates half of the SM's 512 tensor-memory columns)
constexpr int kTcSmemBytes = 80 * 1024;
constexpr long long kTcSpinLimit = 1LL << 24;

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t *bar, int count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)),
                 "r"(count));
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}

// Waits until the phase with the given parity of `bar` has completed, at
// most kTcSpinLimit polls; false (and g_tc_error set) if it never did.
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity) {
    const uint32_t a = smem_u32(bar);
    for (long long it = 0; it < kTcSpinLimit; ++it) {
        uint32_t done;
        asm volatile(
            "{\n\t.reg .pred p;\n\t"
            "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
            "selp.u32 %0, 1, 0, p;\n\t}"
            : "=r"(done)
            : "r"(a), "r"(parity)
            : "memory");
        if (done) return true;
    }
    atomicExch(&g_tc_error, 1);
    return false;
}

__device__ __forceinline__ void tc_fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// kind::tf32, D float32, A and B tf32 K-major, M = 128, N = 16
constexpr uint32_t kTcIdesc = (1u << 4) | (2u << 7) | (2u << 10) |
                              ((uint32_t)(kTcN >> 3) << 17) | ((128u >> 4) << 24);

// shared-memory descriptor of one B slab (no swizzle, K-major)
__device__ __forceinline__ uint64_t b_desc(uint32_t addr) {
    return (uint64_t)((addr >> 4) & 0x3FFF) | ((uint64_t)(128 >> 4) << 16) |
           ((uint64_t)(256 >> 4) << 32) | (1ull << 46);
}

__device__ __forceinline__ void tc_mma(uint32_t d_tmem, uint32_t a_tmem,
                                       uint64_t bdesc, bool accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::tf32 [%0], [%1], %2, %3, p;\n\t}"
        ::"r"(d_tmem), "r"(a_tmem), "l"(bdesc), "r"(kTcIdesc),
        "r"((uint32_t)accumulate)
        : "memory");
}

__device__ __forceinline__ void tc_commit(uint64_t *bar) {
    asm volatile(
        "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
        ::"r"(smem_u32(bar))
        : "memory");
}

// 8 consecutive columns of this warp's 32 lanes
__device__ __forceinline__ void tmem_store8(uint32_t taddr, const uint32_t (&v)[8]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};"
        ::"r"(taddr), "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]),
        "r"(v[5]), "r"(v[6]), "r"(v[7])
        : "memory");
}

__device__ __forceinline__ void tmem_store_wait() {
    asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// 16 consecutive columns of this warp's 32 lanes
__device__ __forceinline__ void tmem_load16(uint32_t taddr, float (&d)[16]) {
    uint32_t r[16];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {"
        "%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]),
          "=r"(r[6]), "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]),
          "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr)
        : "memory");
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 16; ++i) d[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ float2 f2(float v) { return make_float2(v, v); }

// B of chunk c (rows k < 32: the chunk's voxels for the high parts, k >= 32:
// the same voxels for the remainders), phi in half-voxel units about the
// z-quarter's centre. Byte offset of (k, n) in the no-swizzle K-major layout.
__device__ __forceinline__ int b_offset(int c, int k, int n) {
    const int kk = k >> 3, kr = k & 7;
    return c * (2 * kTcChunk / 8) * kTcSlabBytes + kk * kTcSlabBytes +
           (n >> 3) * 256 + (kr >> 2) * 128 + (n & 7) * 16 + (kr & 3) * 4;
}

__device__ float phi(int n, int v) {
    // v = quarter voxel index zl * 64 + y * 8 + x
    const float qx = 2.f * (float)(v & 7) - 7.f;
    const float qy = 2.f * (float)((v >> 3) & 7) - 7.f;
    const float qz = 2.f * (float)(v >> 6) - 1.f;
    switch (n) {
        case 0: return 1.f;
        case 1: return qx;
        case 2: return qy;
        case 3: return qz;
        case 4: return qx * qx;
        case 5: return qy * qy;
        case 7: return qx * qy;
        case 8: return qx * qz;
        case 9: return qy * qz;
        default: return 0.f;
    }
}

struct TcShared {
    uint64_t full[kTcBufs], empty[kTcBufs], dfull[2];
    uint32_t tmem_base;
    float red[2][kTcProducerWarps][kTcPairs][kTcRedStride];
};

// One lane's pair of a pack, as loaded from the pair list and the records.
struct TcPair {
    int gid, tile;
    bool valid;
    float4 r0, r1, r2;
};

__device__ __forceinline__ TcPair load_pair(long long i, long long npairs,
                                            const int *__restrict__ ids,
                                            const int *__restrict__ tile_of,
                                            const float4 *__restrict__ rec) {
    TcPair q;
    q.valid = i < npairs;
    q.gid = 0;
    q.tile = 0;
    q.r0 = make_float4(0.f, 0.f, 0.f, __int_as_float(0x7f800000));
    q.r1 = make_float4(0.f, 0.f, 0.f, 0.f);
    q.r2 = q.r1;
    if (q.valid) {
        q.gid = __ldg(ids + i);
        q.tile = __ldg(tile_of + i);
        q.r0 = __ldg(rec + 3 * (size_t)q.gid);
        q.r1 = __ldg(rec + 3 * (size_t)q.gid + 1);
        q.r2 = __ldg(rec + 3 * (size_t)q.gid + 2);
    }
    return q;
}

// What a pack's epilogue needs of its lane (kept while the next pack runs).
struct TcEpi {
    int gid;
    bool valid;
    float cx, cy, cz, corr, kI;
    float nqa, nqb, nqc, nqd, nqe, nqf;
};

// 32 evaluations of one chunk, stored into the A buffer at `taddr`: alpha *
// g split into tf32 high parts (columns 0..31) and remainders (columns
// 32..63), one 8-voxel row at a time. FLUSH: the cull is the flush to zero
// of ex2 (P carries -(thr + 126)); else the reference's compares.
template <bool FLUSH>
__device__ __forceinline__ void eval_chunk(int c, float my, float mz, float A,
                                           float B, float Cz, float D, float E,
                                           float F, float shift, float thr,
                                           bool robust, const float2 (&dxp)[4],
                                           const float4 (&gv)[8],
                                           uint32_t taddr) {
    const float dz = mz - ((float)(c >> 1) + 0.5f);
    const float Pz = Cz * dz * dz - shift;
#pragma unroll
    for (int yy = 0; yy < 4; ++yy) {
        const float dy = my - ((float)(4 * (c & 1) + yy) + 0.5f);
        const float L = fmaf(D, dy, E * dz);
        const float P = fmaf(dy, fmaf(B, dy, F * dz), Pz);
        uint32_t hv[8], lv[8];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const float2 sp =
                __ffma2_rn(dxp[k], __ffma2_rn(f2(A), dxp[k], f2(L)), f2(P));
            float2 a;
            if (FLUSH) {
                a = make_float2(ex2(sp.x), ex2(sp.y));
            } else {
                const bool ok0 = sp.x >= thr && (robust || sp.x <= 0.f);
                const bool ok1 = sp.y >= thr && (robust || sp.y <= 0.f);
                a = make_float2(ok0 ? ex2(sp.x) : 0.f, ok1 ? ex2(sp.y) : 0.f);
            }
            const float4 gq = gv[2 * yy + (k >> 1)];
            const float2 gg =
                (k & 1) ? make_float2(gq.z, gq.w) : make_float2(gq.x, gq.y);
            const float2 as = __fmul2_rn(a, gg);
            const float2 hi = make_float2(
                __uint_as_float(__float_as_uint(as.x) & 0xFFFFE000u),
                __uint_as_float(__float_as_uint(as.y) & 0xFFFFE000u));
            const float2 lo = __ffma2_rn(hi, f2(-1.f), as);
            hv[2 * k] = __float_as_uint(hi.x);
            hv[2 * k + 1] = __float_as_uint(hi.y);
            lv[2 * k] = __float_as_uint(lo.x);
            lv[2 * k + 1] = __float_as_uint(lo.y);
        }
        tmem_store8(taddr + 8 * yy, hv);
        tmem_store8(taddr + kTcChunk + 8 * yy, lv);
    }
}

__global__ void __launch_bounds__(kTcThreads, 2)
vox_bwd_tc_kernel(Geom g, const int *__restrict__ ids,
                  const int *__restrict__ tile_of,
                  const float4 *__restrict__ rec,
                  const float *__restrict__ sign_plane,
                  const long long *__restrict__ pair_total, long long pair_cap,
                  float *__restrict__ pos_grad, float *__restrict__ conic_grad,
                  float *__restrict__ int_grad,
                  const float *__restrict__ grad_loss, float inv_denom) {
    extern __shared__ __align__(1024) unsigned char tc_smem_raw[];
    // B first (1 KB aligned), then the barriers and reduction buffers
    unsigned char *bsm = tc_smem_raw;
    TcShared &S = *reinterpret_cast<TcShared *>(tc_smem_raw + kTcBBytes);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const bool mma_warp = warp == kTcProducerWarps;

    // constant B: 4 chunks x 64 rows x 16 columns
    for (int e = threadIdx.x; e < kTcChunks * 2 * kTcChunk * kTcN; e += blockDim.x) {
        const int n = e % kTcN, k = (e / kTcN) % (2 * kTcChunk),
                  c = e / (kTcN * 2 * kTcChunk);
        const int v = c * kTcChunk + (k & (kTcChunk - 1));
        *reinterpret_cast<float *>(bsm + b_offset(c, k, n)) = phi(n, v);
    }
    if (threadIdx.x == 0) {
        for (int b = 0; b < kTcBufs; ++b) {
            mbar_init(&S.full[b], kTcProducerWarps);
            mbar_init(&S.empty[b], 1);
        }
        mbar_init(&S.dfull[0], 1);
        mbar_init(&S.dfull[1], 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    // B is read by the tensor cores (async proxy)
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    if (mma_warp) {
        asm volatile(
            "tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
            ::"r"(smem_u32(&S.tmem_base)), "r"(kTcCols)
            : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tbase = S.tmem_base;

    const long long total = *pair_total;
    const long long npairs = total < pair_cap ? total : pair_cap;
    const long long packs = (npairs + kTcPairs - 1) / kTcPairs;
    const float scale = (*grad_loss) * inv_denom;
    bool ok = true;

    if (mma_warp) {
        // ---------------------------------------------------- MMA issuer
        // pack t accumulates into D buffer t & 1; chunk n uses A buffer
        // n % kTcBufs
        const uint32_t bbase = smem_u32(bsm);
        long long n = 0, t = 0;
        if (lane == 0) {
            for (long long p = blockIdx.x; p < packs && ok; p += gridDim.x, ++t) {
                const uint32_t dcol = tbase + kTcDCol + (uint32_t)((t & 1) * kTcN);
                for (int c = 0; c < kTcChunks && ok; ++c, ++n) {
                    const int b = (int)(n % kTcBufs);
                    ok = mbar_wait(&S.full[b], (uint32_t)((n / kTcBufs) & 1));
                    if (!ok) break;
                    tc_fence_after();
                    const uint32_t a0 = tbase + (uint32_t)(b * kTcBufCols);
#pragma unroll
                    for (int kk = 0; kk < 2 * kTcChunk / 8; ++kk)
                        tc_mma(dcol, a0 + 8 * kk,
                               b_desc(bbase + c * (2 * kTcChunk / 8) * kTcSlabBytes +
                                      kk * kTcSlabBytes),
                               c > 0 || kk > 0);
                    tc_commit(&S.empty[b]);
                    if (c == kTcChunks - 1) tc_commit(&S.dfull[t & 1]);
                }
            }
            // the last pack's MMAs have completed before the memory is freed
            if (t > 0 && ok) mbar_wait(&S.dfull[(t - 1) & 1], (uint32_t)(((t - 1) >> 1) & 1));
        }
        __syncwarp();
    } else {
        // ------------------------------------------------------ producers
        const int u = warp;  // z-quarter of this warp's rows
        const uint32_t lane_addr = tbase + ((uint32_t)(32 * u) << 16);
        long long n = 0, t = 0;
        TcEpi prev;
        prev.valid = false;
        prev.gid = 0;
        long long p = blockIdx.x;
        TcPair cur = load_pair(p * kTcPairs + lane, npairs, ids, tile_of, rec);

        // Moments of pack tt (D buffer tt & 1) -> the pair's gradients.
        auto epilogue = [&](long long tt, const TcEpi &E) {
            if (ok) ok = mbar_wait(&S.dfull[tt & 1], (uint32_t)((tt >> 1) & 1));
            ok = __all_sync(0xffffffffu, ok);
            tc_fence_after();
            float M[16];
            tmem_load16(lane_addr + kTcDCol + (uint32_t)((tt & 1) * kTcN), M);
            // sums about the Gaussian centre: d = c - q / 2 with c the centre
            // relative to the quarter's centre (4, 4, 1)
            const float cx = E.cx, cy = E.cy, cz = E.cz, m0 = M[0];
            float sm[kTcSums];
            sm[0] = fmaf(cx, m0, -0.5f * M[1]);                   // Vx
            sm[1] = fmaf(cy, m0, -0.5f * M[2]);                   // Vy
            sm[2] = fmaf(cz, m0, -0.5f * M[3]);                   // Vz
            sm[3] = fmaf(cx, fmaf(cx, m0, -M[1]), 0.25f * M[4]);  // Sxx
            sm[4] = fmaf(cy, fmaf(cy, m0, -M[2]), 0.25f * M[5]);  // Syy
            sm[5] = fmaf(cz, fmaf(cz, m0, -M[3]), 0.25f * m0);    // Szz
            sm[6] = fmaf(cx * cy, m0, fmaf(-0.5f, fmaf(cx, M[2], cy * M[1]), 0.25f * M[7]));
            sm[7] = fmaf(cx * cz, m0, fmaf(-0.5f, fmaf(cx, M[3], cz * M[1]), 0.25f * M[8]));
            sm[8] = fmaf(cy * cz, m0, fmaf(-0.5f, fmaf(cy, M[3], cz * M[2]), 0.25f * M[9]));
            sm[9] = m0;                                           // W
            float(&red)[kTcProducerWarps][kTcPairs][kTcRedStride] = S.red[tt & 1];
#pragma unroll
            for (int k = 0; k < kTcSums; ++k) red[u][lane][k] = sm[k] * E.corr;
            // the four quarters of each pair meet in warp 0
            asm volatile("bar.sync 1, %0;" ::"r"(kTcProducerWarps * 32) : "memory");
            if (u == 0 && E.valid) {
                float ts[kTcSums];
#pragma unroll
                for (int k = 0; k < kTcSums; ++k)
                    ts[k] = red[0][lane][k] + red[1][lane][k] + red[2][lane][k] +
                            red[3][lane][k];
                const float kI = E.kI;  // sigma_grad = I * w
                const float vx = kI * ts[0], vy = kI * ts[1], vz = kI * ts[2];
                red_add4(pos_grad + 4 * (size_t)E.gid,
                         E.nqa * vx + E.nqb * vy + E.nqc * vz,
                         E.nqb * vx + E.nqd * vy + E.nqe * vz,
                         E.nqc * vx + E.nqe * vy + E.nqf * vz, 0.f);
                float *cg = conic_grad + 6 * (size_t)E.gid;
                red_add2(cg + 0, -0.5f * kI * ts[3], -kI * ts[6]);
                red_add2(cg + 2, -kI * ts[7], -0.5f * kI * ts[4]);
                red_add2(cg + 4, -kI * ts[8], -0.5f * kI * ts[5]);
                red_add(int_grad + E.gid, ts[9]);
            }
            // red[tt & 1] is written again by pack tt + 2's epilogue, after
            // that pack's MMAs, which need warp 0's chunks of pack tt + 2,
            // issued after warp 0 has read it here
        };

        for (; p < packs; p += gridDim.x, ++t) {
            // the next pack's pair data, in flight during this pack
            const TcPair nxt = load_pair((p + gridDim.x) * kTcPairs + lane, npairs,
                                         ids, tile_of, rec);
            const int tx = cur.tile % g.Tx, rest = cur.tile / g.Tx;
            const int ty = rest % g.Ty, tz = rest / g.Ty + g.tz0;
            // centre relative to voxel (0,0,0) of this z-quarter
            const float mx = cur.r0.x - (float)(tx * kTile);
            const float my = cur.r0.y - (float)(ty * kTile);
            const float mz = cur.r0.z - (float)(tz * kTile + 2 * u);
            const float thr = cur.r0.w;
            const bool robust = (__float_as_uint(thr) & 1u) != 0u;
            const bool flush =
                __all_sync(0xffffffffu, !cur.valid || (robust && thr >= -126.f));
            const float shift = flush ? thr + 126.f : 0.f;
            const float A = cur.r1.x, B = cur.r1.y, Cz = cur.r1.z, D = cur.r1.w,
                        E = cur.r2.x, F = cur.r2.y;
            float2 dxp[4];
#pragma unroll
            for (int k = 0; k < 4; ++k)
                dxp[k] = make_float2(mx - (2.f * k + 0.5f), mx - (2.f * k + 1.5f));
            const float4 *gp = reinterpret_cast<const float4 *>(
                sign_plane + (size_t)cur.tile * kTileVoxels + u * (kTileVoxels / 4));
            float4 gv[8];
#pragma unroll
            for (int q = 0; q < 8; ++q)
                gv[q] = cur.valid ? __ldg(gp + q) : make_float4(0.f, 0.f, 0.f, 0.f);

            for (int c = 0; c < kTcChunks; ++c, ++n) {
                float4 gn[8];  // next chunk's signs, in flight
#pragma unroll
                for (int q = 0; q < 8; ++q)
                    gn[q] = (cur.valid && c + 1 < kTcChunks)
                                ? __ldg(gp + (c + 1) * 8 + q)
                                : make_float4(0.f, 0.f, 0.f, 0.f);
                const int b = (int)(n % kTcBufs);
                const long long use = n / kTcBufs;
                if (use > 0 && ok) ok = mbar_wait(&S.empty[b], (uint32_t)((use - 1) & 1));
                ok = __all_sync(0xffffffffu, ok);
                const uint32_t abuf = lane_addr + (uint32_t)(b * kTcBufCols);
                if (flush)
                    eval_chunk<true>(c, my, mz, A, B, Cz, D, E, F, shift, thr,
                                     robust, dxp, gv, abuf);
                else
                    eval_chunk<false>(c, my, mz, A, B, Cz, D, E, F, shift, thr,
                                      robust, dxp, gv, abuf);
                tmem_store_wait();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&S.full[b]);
#pragma unroll
                for (int q = 0; q < 8; ++q) gv[q] = gn[q];
            }
            // the previous pack's epilogue overlaps this pack's MMAs
            if (t > 0) epilogue(t - 1, prev);
            prev.valid = cur.valid;
            prev.gid = cur.gid;
            prev.cx = mx - 4.f;
            prev.cy = my - 4.f;
            prev.cz = mz - 1.f;
            // (a pair whose every voxel was culled has zero sums; the clamp
            // keeps 0 * corr finite)
            prev.corr = scale * ex2(fminf(shift - 64.f, 127.f));
            prev.kI = cur.r2.z;
            prev.nqa = 2.f * kLn2 * cur.r1.x;
            prev.nqd = 2.f * kLn2 * cur.r1.y;
            prev.nqf = 2.f * kLn2 * cur.r1.z;
            prev.nqb = kLn2 * cur.r1.w;
            prev.nqc = kLn2 * cur.r2.x;
            prev.nqe = kLn2 * cur.r2.y;
            cur = nxt;
        }
        if (t > 0) epilogue(t - 1, prev);
    }
    tc_fence_before();
    __syncthreads();
    if (mma_warp) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;"
                     ::"r"(tbase), "r"(kTcCols)
                     : "memory");
    }
}

}  // namespace

// Grid: two CTAs per SM (each holds half of the tensor memory).
cudaError_t launch_vox_backward_tc(const Geom &g, const int *ids,
                                   const int *tile_of, const float4 *rec,
                                   const float *sign_plane,
                                   const long long *pair_total,
                                   long long pair_cap, float *pos_grad,
                                   float *conic_grad, float *int_grad,
                                   const float *grad_loss, float inv_denom,
                                   cudaStream_t stream) {
    static int grid = 0;
    if (grid == 0) {
        cudaError_t err = cudaFuncSetAttribute(
            vox_bwd_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
            kTcSmemBytes);
        if (err) return err;
        int dev = 0, sms = kSMs;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
        grid = 2 * sms;
    }
    static_assert(kTcBBytes + sizeof(TcShared) <= kTcSmemBytes, "smem");
    static_assert(kTcDCol + 2 * kTcN <= kTcCols, "tensor memory");
    vox_bwd_tc_kernel<<<grid, kTcThreads, kTcSmemBytes, stream>>>(
        g, ids, tile_of, rec, sign_plane, pair_total, pair_cap, pos_grad,
        conic_grad, int_grad, grad_loss, inv_denom);
    count_launches(1);
    return cudaGetLastError();
}

int tc_error_flag(bool clear) {
    int v = 0;
    if (cudaMemcpyFromSymbol(&v, g_tc_error, sizeof(int)) != cudaSuccess) return -1;
    if (clear && v) {
        const int zero = 0;
        if (cudaMemcpyToSymbol(g_tc_error, &zero, sizeof(int)) != cudaSuccess)
            return -1;
    }
    return v;
}

}  // namespace gsv
