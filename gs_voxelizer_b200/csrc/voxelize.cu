// Forward and backward voxelization of 3D Gaussians on 8x8x8 voxel tiles.
//
// Semantics follow gs_voxelizer/cuda/voxelize.cu of the reference:
//   forward  :39-164   vol[v] = sum_g I_g * exp(sigma_g(v)) over the tile's
//                      Gaussians, sigma = -1/2 d^T Q d, d = mu - (voxel+0.5),
//                      skipping sigma > 0 / non-finite and alpha*mean(I)<1e-6
//   backward :170-366 (per voxel) and :368-574 (per Gaussian): gradients of
//                      the same sum w.r.t. mu, the six conic entries and I.
//
// The arithmetic is reorganised for the SM's issue rate (one warp
// instruction per SMSP per clock; MUFU.EX2 at 16/clk/SM):
//   * A per-Gaussian record is built once per call: centre, the conic scaled
//     by log2(e) so that one ex2 gives exp(sigma), and the alpha*mean(I)
//     cull rewritten as a threshold on the log2 exponent (s >= thr).
//   * sigma along a line of 8 voxels in z is a quadratic P + L*dz + C*dz^2;
//     P and L are formed once per (Gaussian, column), so an evaluation costs
//     two FMAs and one ex2 - executed as paired FP32 instructions
//     (FFMA2/FMUL2/FADD2), two evaluations per instruction.
//   * The cull costs no compare for robustly positive-definite Gaussians
//     with -126 <= thr <= -1: the forward multiplies alpha by 2^(-thr-126)
//     with a flush-to-zero multiply (exactly 0 below the threshold) and
//     accumulates with I * 2^(thr+126); the backward evaluates
//     ex2(s - thr - 126), flushed to 0 by ex2.approx.ftz, on a dL/dvol tile
//     staged x 2^K and rescales each Gaussian's sums once. Other Gaussians
//     take the exact compare path.
//   * Forward: exponentials by recurrence along z (two ex2 anchors per
//     column of 8) where the anchor provably never underflows.
//   * "sigma > 0" can only happen for a conic that is not positive definite
//     or is so ill-conditioned that rounding flips the sign. The record marks
//     Gaussians whose conic satisfies det(Q) >= 1e-5 trace(Q)^3 (so
//     lambda_min / lambda_max >= 1e-5, far above the rounding error of the
//     6-term quadratic); for them the test provably never fires and is
//     skipped. Other Gaussians take the fully checked path.
//   * Backward sums are factored: along a z column only sum(w), sum(w dz) and
//     sum(w dz^2) are accumulated (w = alpha * dL/dvol); the six conic and
//     three position sums are rebuilt from them with the column's dx, dy.
#include "common.cuh"

namespace gsv {

cudaError_t scan_counts_to_bins(int *counts, long long ntiles,
                                long long *partials, int *tile_bins,
                                cudaStream_t stream, long long cap,
                                long long *count_out = nullptr,
                                float *overflow_out = nullptr,
                                const ItemScan *items = nullptr);
cudaError_t launch_vox_backward_tc(const Geom &g, const int *ids,
                                   const int *tile_of, const float4 *rec,
                                   const float *sign_plane,
                                   const long long *pair_total,
                                   long long pair_cap, float *pos_grad,
                                   float *conic_grad, float *int_grad,
                                   const float *grad_loss, float inv_denom,
                                   cudaStream_t stream);
size_t l1_workspace_bytes(long long n);
cudaError_t launch_sum(long long n, const float *a, const float *b,
                       double inv_denom, float *out, void *ws,
                       cudaStream_t stream);

namespace {

constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;

template <int C>
struct Rec {
    static constexpr int kF4 = C <= 2 ? 3 : 4;  // float4 per record
};

__device__ __forceinline__ bool robust_flag(float thr) {
    return (__float_as_uint(thr) & 1u) != 0u;
}

// record: r0 = (mx, my, mz, thr), r1 = (A, B, Cz, D), r2 = (E, F, I0, I1),
//         r3 = (I2, I3, 0, 0)  with
// s = A dx^2 + B dy^2 + Cz dz^2 + D dx dy + E dx dz + F dy dz = log2(e) sigma.
// The lowest mantissa bit of thr carries the "robustly positive definite"
// flag (1 ulp of the threshold; the cull is already approximate there).
template <int C>
__global__ void __launch_bounds__(256)
prep_records_kernel(int n, const float4 *__restrict__ pos_radii,
                    const float2 *__restrict__ conics,
                    const float *__restrict__ intensities,
                    float4 *__restrict__ rec) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    constexpr int R = Rec<C>::kF4;
    const float4 p = pos_radii[i];
    const float2 ab = conics[3 * i + 0], cd = conics[3 * i + 1],
                 ef = conics[3 * i + 2];
    float I[4] = {0.f, 0.f, 0.f, 0.f};
    float mean = 0.f;
#pragma unroll
    for (int c = 0; c < C; ++c) {
        I[c] = intensities[i * C + c];
        mean += I[c];
    }
    mean /= C;
    float thr;
    if (mean > 0.f) {
        thr = (float)log2((double)0.000001f / (double)mean);
    } else if (mean <= 0.f) {
        thr = __int_as_float(0x7f800000);  // +inf: never contributes
    } else {
        thr = __int_as_float(0xff800000);  // NaN mean: -inf, output is NaN
    }
    // robust positive definiteness of Q = [[a b c][b d e][c e f]]
    const double a = ab.x, b = ab.y, c = cd.x, d = cd.y, e = ef.x, f = ef.y;
    const double m2 = a * d - b * b;
    const double det = a * (d * f - e * e) - b * (b * f - e * c) +
                       c * (b * e - d * c);
    const double tr = a + d + f;
    const bool robust = a > 0.0 && m2 > 0.0 && det > 0.0 &&
                        det >= 1e-5 * tr * tr * tr && isfinite(det) &&
                        isfinite(tr);
    if (isfinite(thr)) {
        unsigned bits = __float_as_uint(thr);
        bits = robust ? (bits | 1u) : (bits & ~1u);
        thr = __uint_as_float(bits);
    }
    const float h = -0.5f * kLog2e;
    rec[i * R + 0] = make_float4(p.x, p.y, p.z, thr);
    rec[i * R + 1] =
        make_float4(h * ab.x, h * cd.y, h * ef.y, -kLog2e * ab.y);
    rec[i * R + 2] = make_float4(-kLog2e * cd.x, -kLog2e * ef.x, I[0], I[1]);
    if (R == 4) rec[i * R + 3] = make_float4(I[2], I[3], 0.f, 0.f);
}

__device__ __forceinline__ void tile_coords(const Geom &g, long long tile,
                                            int &ox, int &oy, int &oz) {
    const int tx = (int)(tile % g.Tx);
    const long long rest = tile / g.Tx;
    const int ty = (int)(rest % g.Ty);
    const int tz = (int)(rest / g.Ty) + g.tz0;
    ox = tx * kTile;
    oy = ty * kTile;
    oz = tz * kTile;
}

template <int C>
__device__ __forceinline__ void record_intensity(const float4 &r2,
                                                 const float4 &r3,
                                                 float (&I)[C]) {
    I[0] = r2.z;
    if (C > 1) I[1 % C] = r2.w;
    if (C > 2) I[2 % C] = r3.x;
    if (C > 3) I[3 % C] = r3.y;
}

// ---------------------------------------------------------------- forward
//
// One warp per tile. Lane (x, y) with x = lane & 7, y = lane >> 3 owns the
// two z-columns (x, y) and (x, y + 4): 16 voxels. Gaussian records are
// staged in shared memory in batches, tile-relative, together with the eight
// z-offsets dz_j = mz - (j + 0.5) every lane needs.

constexpr int kFwdBatch = 64;

// acc += I * a when thr <= s (and s <= 0 when CHECK_SIGN): one compare and
// one predicated FMA.
template <bool CHECK_SIGN>
__device__ __forceinline__ void fma_if_valid(float &acc, float I, float a,
                                             float s, float thr) {
    if (CHECK_SIGN) {
        asm("{\n\t.reg .pred p;\n\t"
            "setp.ge.f32 p, %1, %2;\n\t"
            "setp.le.and.f32 p, %1, 0f00000000, p;\n\t"
            "@p fma.rn.f32 %0, %3, %4, %0;\n\t}"
            : "+f"(acc) : "f"(s), "f"(thr), "f"(I), "f"(a));
    } else {
        asm("{\n\t.reg .pred p;\n\t"
            "setp.ge.f32 p, %1, %2;\n\t"
            "@p fma.rn.f32 %0, %3, %4, %0;\n\t}"
            : "+f"(acc) : "f"(s), "f"(thr), "f"(I), "f"(a));
    }
}

__device__ __forceinline__ float2 f2(float v) { return make_float2(v, v); }

// sign(d) as -1, 0 or 1 (0 for NaN, as the L1 gradient's staging treats it)
__device__ __forceinline__ float sign_of(float d) {
    return d > 0.f ? 1.f : (d < 0.f ? -1.f : 0.f);
}

// sigma (log2 units) of the lane's two columns at z-offset dz:
// s = P + dz * (L + Cz * dz), evaluated as paired FP32 FMAs (FFMA2).
__device__ __forceinline__ float2 sigma_pair(float2 P, float2 L, float Cz,
                                             float dz) {
    const float2 d = f2(dz);
    return __ffma2_rn(d, __ffma2_rn(f2(Cz), d, L), P);
}

// Accumulators acc[j][c] hold the lane's two columns, (x, y) in .x and
// (x, y + 4) in .y, at z-offset j, so that they update as pairs.

// Exact path: acc += I * alpha where thr <= s (and s <= 0 when CHECK_SIGN),
// one compare and one predicated FMA per evaluation.
template <int C, bool CHECK_SIGN>
__device__ __forceinline__ void fwd_accumulate(float2 (&acc)[8][C], int j,
                                               const float (&I)[C], float a0,
                                               float a1, float s0, float s1,
                                               float thr) {
    if (C == 1) {
        fma_if_valid<CHECK_SIGN>(acc[j][0].x, I[0], a0, s0, thr);
        fma_if_valid<CHECK_SIGN>(acc[j][0].y, I[0], a1, s1, thr);
    } else {
        bool ok0 = s0 >= thr, ok1 = s1 >= thr;
        if (CHECK_SIGN) {
            ok0 &= s0 <= 0.f;
            ok1 &= s1 <= 0.f;
        }
#pragma unroll
        for (int c = 0; c < C; ++c) {
            if (ok0) acc[j][c].x = fmaf(I[c], a0, acc[j][c].x);
            if (ok1) acc[j][c].y = fmaf(I[c], a1, acc[j][c].y);
        }
    }
}

// Flush path (robustly positive-definite Gaussians, -126 <= thr <= -1):
// m = alpha * cm with cm = 2^(-thr - 126) is below the smallest normal
// float, and flushed to exactly 0, precisely when alpha < 2^thr (the cull);
// acc += m * Is with Is = I * 2^(thr + 126) restores the scale. Two
// evaluations per paired instruction, no compare.
template <int C>
__device__ __forceinline__ void fwd_accumulate_flush(float2 (&acc)[8][C],
                                                     int j,
                                                     const float2 (&Is)[C],
                                                     float2 a, float2 cm) {
    const float2 m = fmul2_ftz(a, cm);
#pragma unroll
    for (int c = 0; c < C; ++c) acc[j][c] = ffma2_ftz(m, Is[c], acc[j][c]);
}

// One exponential per evaluation, exact cull.
template <int C, bool CHECK_SIGN>
__device__ __forceinline__ void fwd_pair_direct(float2 P, float2 L, float Cz,
                                                float thr,
                                                const float (&dz)[8],
                                                const float (&I)[C],
                                                float2 (&acc)[8][C]) {
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        const float2 s = sigma_pair(P, L, Cz, dz[j]);
        fwd_accumulate<C, CHECK_SIGN>(acc, j, I, ex2(s.x), ex2(s.y), s.x, s.y,
                                      thr);
    }
}

// One exponential per evaluation, flush-mask cull.
template <int C>
__device__ __forceinline__ void fwd_pair_direct_flush(float2 P, float2 L,
                                                      float Cz, float2 cm,
                                                      const float (&dz)[8],
                                                      const float2 (&Is)[C],
                                                      float2 (&acc)[8][C]) {
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        const float2 s = sigma_pair(P, L, Cz, dz[j]);
        fwd_accumulate_flush<C>(acc, j, Is, make_float2(ex2(s.x), ex2(s.y)),
                                cm);
    }
}

// Exponentials by recurrence along z. With dz_{j+1} = dz_j - 1 the exponent
// steps by D_j = s_{j+1} - s_j and D_{j+1} = D_j + 2 Cz, so
//   alpha_{j+1} = alpha_j * r_j,  r_{j+1} = r_j * q,  q = 2^(2 Cz).
// Two anchors (j = 0 and j = 4) each start a 4-point chain: 4 ex2 per 8
// voxels instead of 8. Only used when |Cz| <= 2 and thr >= -40: then any
// point of a chain above the cull threshold implies the chain's anchor
// exponent is >= -112 (concave quadratic, slope <= 2 sqrt(40 |Cz|)), so the
// anchor never flushes to zero while a later point still counts, and the
// products stay within ~10 ulp of the direct exponential. The chain runs
// on unscaled alpha; the cull is the flush mask of fwd_accumulate_flush.
template <int C>
__device__ __forceinline__ void fwd_pair_chain(float2 P, float2 L, float Cz,
                                               float q, float2 cm,
                                               const float (&dz)[8],
                                               const float2 (&Is)[C],
                                               float2 (&acc)[8][C]) {
#pragma unroll
    for (int seg = 0; seg < 8; seg += 4) {
        const float2 s0 = sigma_pair(P, L, Cz, dz[seg]);
        const float2 s1 = sigma_pair(P, L, Cz, dz[seg + 1]);
        const float2 d = __ffma2_rn(s0, f2(-1.f), s1);
        float2 a = make_float2(ex2(s0.x), ex2(s0.y));
        // s <= 0 (robust), so a step ratio above 2^126 only follows an
        // anchor that flushed to 0; the clamp keeps that chain at 0 * finite
        // (the flush mask does not discard NaN as a compare would)
        float2 r = make_float2(ex2(fminf(d.x, 126.f)), ex2(fminf(d.y, 126.f)));
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            if (k > 0) {
                a = __fmul2_rn(a, r);
                if (k < 3) r = __fmul2_rn(r, f2(q));
            }
            fwd_accumulate_flush<C>(acc, seg + k, Is, a, cm);
        }
    }
}

// LOSS: also reduce sum |vol - target| over the tile's voxels into
// tile_loss[tile] (the fused L1 loss; target has the output's layout).
template <int C, bool LOSS>
__global__ void __launch_bounds__(32, C <= 2 ? 32 : 16)
vox_fwd_kernel(Geom g, const int2 *__restrict__ bins,
               const int *__restrict__ ids, const float4 *__restrict__ rec,
               float *__restrict__ out, const float *__restrict__ target,
               float *__restrict__ tile_loss, float *__restrict__ sign_plane,
               int *__restrict__ tile_of) {
    constexpr int R = Rec<C>::kF4;
    // record + 8 dz + (q, cm, mode, 1 / cm), padded to 7 float4 (112 B):
    // with a 28-word stride the eight float4 stores of a quarter-warp hit
    // eight different bank groups
    constexpr int RS = 7;
    constexpr int kStage = (kFwdBatch * RS * 4 > kTileVoxels * C)
                               ? kFwdBatch * RS * 4
                               : kTileVoxels * C;
    __shared__ __align__(16) float smem[kStage];
    float4 *sb = reinterpret_cast<float4 *>(smem);

    const long long tile = blockIdx.x;
    int ox, oy, oz;
    tile_coords(g, tile, ox, oy, oz);
    const int lane = threadIdx.x;
    const int lx = lane & 7, ly = lane >> 3;
    const float fx = lx + 0.5f, fy = ly + 0.5f;

    float2 acc[8][C];
#pragma unroll
    for (int j = 0; j < 8; ++j)
#pragma unroll
        for (int c = 0; c < C; ++c) acc[j][c] = make_float2(0.f, 0.f);

    const int2 range = bins[tile];
    if (tile_of) {  // the tile of every pair, for the tensor-core backward
        for (int k = range.x + lane; k < range.y; k += 32) tile_of[k] = (int)tile;
    }
    for (int s0 = range.x; s0 < range.y; s0 += kFwdBatch) {
        const int nb = min(kFwdBatch, range.y - s0);
        __syncwarp();
        for (int k = lane; k < nb; k += 32) {
            const int gid = ids[s0 + k];
            float4 r0 = rec[(size_t)gid * R];
            r0.x -= (float)ox;
            r0.y -= (float)oy;
            r0.z -= (float)oz;
            sb[k * RS] = r0;
#pragma unroll
            for (int q = 1; q < R; ++q) sb[k * RS + q] = rec[(size_t)gid * R + q];
            sb[k * RS + R] = make_float4(r0.z - 0.5f, r0.z - 1.5f, r0.z - 2.5f,
                                         r0.z - 3.5f);
            sb[k * RS + R + 1] = make_float4(r0.z - 4.5f, r0.z - 5.5f,
                                             r0.z - 6.5f, r0.z - 7.5f);
            // per-Gaussian mode: 2 chain + flush mask, 1 direct + flush
            // mask, 0 exact compare (not robust, or thr out of range)
            const float Cz = sb[k * RS + 1].z, thr = r0.w;
            const bool flush =
                robust_flag(thr) && thr >= -126.f && thr <= -1.f;
            const bool chain = flush && Cz >= -2.f && thr >= -40.f;
            const float cm = flush ? ex2(-thr - 126.f) : 0.f;
            sb[k * RS + R + 2] =
                make_float4(ex2(2.f * Cz), cm, chain ? 2.f : (flush ? 1.f : 0.f),
                            flush ? 1.f / cm : 0.f);
        }
        __syncwarp();
#pragma unroll 1
        for (int t = 0; t < nb; ++t) {
            const float4 r0 = sb[t * RS + 0];
            const float4 r1 = sb[t * RS + 1];
            const float4 r2 = sb[t * RS + 2];
            const float4 r3 = (R == 4) ? sb[t * RS + 3] : r2;
            const float4 za = sb[t * RS + R], zb = sb[t * RS + R + 1];
            const float4 ex = sb[t * RS + R + 2];
            const float dz[8] = {za.x, za.y, za.z, za.w, zb.x, zb.y, zb.z, zb.w};
            float I[C];
            record_intensity<C>(r2, r3, I);
            // P, L of the columns (x, y) and (x, y + 4), as pairs
            const float dx = r0.x - fx;
            const float2 dy = make_float2(r0.y - fy, r0.y - fy - 4.f);
            const float2 P = __ffma2_rn(
                f2(dx), __ffma2_rn(f2(r1.w), dy, f2(r1.x * dx)),
                __fmul2_rn(__fmul2_rn(f2(r1.y), dy), dy));
            const float2 L = __ffma2_rn(f2(r2.y), dy, f2(r2.x * dx));
            if (ex.z != 0.f) {
                float2 Is[C];
#pragma unroll
                for (int c = 0; c < C; ++c) Is[c] = f2(I[c] * ex.w);
                if (ex.z == 2.f)
                    fwd_pair_chain<C>(P, L, r1.z, ex.x, f2(ex.y), dz, Is, acc);
                else
                    fwd_pair_direct_flush<C>(P, L, r1.z, f2(ex.y), dz, Is, acc);
            } else if (robust_flag(r0.w))
                fwd_pair_direct<C, false>(P, L, r1.z, r0.w, dz, I, acc);
            else
                fwd_pair_direct<C, true>(P, L, r1.z, r0.w, dz, I, acc);
        }
    }

    // stage the 8x8x8xC block and store it row by row (x fastest)
    __syncwarp();
#pragma unroll
    for (int k = 0; k < 2; ++k)
#pragma unroll
        for (int j = 0; j < 8; ++j)
#pragma unroll
            for (int c = 0; c < C; ++c)
                smem[((j * 64) + (ly + 4 * k) * 8 + lx) * C + c] =
                    k == 0 ? acc[j][c].x : acc[j][c].y;
    __syncwarp();
    const bool vec_ok = ((reinterpret_cast<uintptr_t>(out) & 15) == 0) &&
                        (!LOSS || (reinterpret_cast<uintptr_t>(target) & 15) == 0);
    float lsum = 0.f;
    if (C == 1 && vec_ok && oz + kTile <= g.z_end() && oy + kTile <= g.Y &&
        ox + kTile <= g.X && (g.X & 3) == 0) {
        // interior tile, one channel: lane l takes float4 l + 32 h of the
        // staged block (rows of 8 voxels, two float4 each), so consecutive
        // lanes read consecutive shared-memory words
        float4 *sp4 = (LOSS && sign_plane)
                          ? reinterpret_cast<float4 *>(sign_plane + (size_t)tile * kTileVoxels)
                          : nullptr;
        constexpr float kSign = 18446744073709551616.f;  // 2^64
#pragma unroll
        for (int h = 0; h < 4; ++h) {
            const int f = lane + 32 * h;       // float4 index in the block
            const int row = f >> 1, q = f & 1;  // row = 8 z + y
            const int z = oz + (row >> 3), y = oy + (row & 7);
            const size_t base =
                ((size_t)(z - g.z_begin()) * g.Y + y) * g.X + ox + 4 * q;
            const float4 v = reinterpret_cast<const float4 *>(smem)[f];
            *reinterpret_cast<float4 *>(out + base) = v;
            if (LOSS) {
                const float4 t = __ldg(reinterpret_cast<const float4 *>(target + base));
                lsum += fabsf(v.x - t.x) + fabsf(v.y - t.y) + fabsf(v.z - t.z) +
                        fabsf(v.w - t.w);
                if (sp4)
                    sp4[f] = make_float4(sign_of(v.x - t.x) * kSign,
                                         sign_of(v.y - t.y) * kSign,
                                         sign_of(v.z - t.z) * kSign,
                                         sign_of(v.w - t.w) * kSign);
            }
        }
        if (LOSS) {
#pragma unroll
            for (int o = 16; o > 0; o >>= 1)
                lsum += __shfl_xor_sync(0xffffffffu, lsum, o);
            if (lane == 0) tile_loss[tile] = lsum;
        }
        return;
    }
    // sign plane (C = 1, fused L1): sign(vol - target) * 2^64 per voxel of
    // the tile, tile-major [z][y][x], 0 outside the volume
    float4 *sp4 = (LOSS && C == 1 && sign_plane)
                      ? reinterpret_cast<float4 *>(sign_plane + (size_t)tile * kTileVoxels)
                      : nullptr;
    constexpr float kSign = 18446744073709551616.f;  // 2^64
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        const int row = lane + 32 * h;  // 64 rows = 8 z * 8 y
        const int z = oz + (row >> 3), y = oy + (row & 7);
        if (sp4 && !(z < g.z_end() && y < g.Y)) {
            sp4[2 * row] = make_float4(0.f, 0.f, 0.f, 0.f);
            sp4[2 * row + 1] = make_float4(0.f, 0.f, 0.f, 0.f);
        }
        if (z < g.z_end() && y < g.Y) {
            const int nx = min(kTile, g.X - ox);
            const size_t base =
                (((size_t)(z - g.z_begin()) * g.Y + y) * g.X + ox) * C;
            const float *src = smem + row * 8 * C;
            float *dst = out + base;
            if (nx == kTile && ((base & 3) == 0) && vec_ok) {
#pragma unroll
                for (int q = 0; q < 2 * C; ++q) {
                    const float4 v = reinterpret_cast<const float4 *>(src)[q];
                    reinterpret_cast<float4 *>(dst)[q] = v;
                    if (LOSS) {
                        const float4 t = __ldg(
                            reinterpret_cast<const float4 *>(target + base) + q);
                        lsum += fabsf(v.x - t.x) + fabsf(v.y - t.y) +
                                fabsf(v.z - t.z) + fabsf(v.w - t.w);
                        if (sp4)
                            sp4[2 * row + q] = make_float4(
                                sign_of(v.x - t.x) * kSign, sign_of(v.y - t.y) * kSign,
                                sign_of(v.z - t.z) * kSign, sign_of(v.w - t.w) * kSign);
                    }
                }
            } else {
                for (int q = 0; q < nx * C; ++q) {
                    dst[q] = src[q];
                    if (LOSS) lsum += fabsf(src[q] - __ldg(target + base + q));
                }
                if (sp4) {
                    float *sp = sign_plane + (size_t)tile * kTileVoxels + row * 8;
                    for (int q = 0; q < 8; ++q)
                        sp[q] = q < nx ? sign_of(src[q] - __ldg(target + base + q)) * kSign
                                       : 0.f;
                }
            }
        }
    }
    if (LOSS) {
#pragma unroll
        for (int o = 16; o > 0; o >>= 1)
            lsum += __shfl_xor_sync(0xffffffffu, lsum, o);
        if (lane == 0) tile_loss[tile] = lsum;
    }
}

// --------------------------------------------------- backward (per Gaussian)
//
// Work item = (tile, bucket of up to 32 consecutive Gaussians of the tile's
// sorted list). A warp takes one item at a time from a global counter. When a
// bucket has m <= 16 Gaussians the warp splits the tile's 8 y-rows into
// r = 2, 4 or 8 groups and gives each lane one (Gaussian, row group), so lanes
// stay busy; the group partials are summed with shuffles before the atomics.
// The tile's dL/dvol block is staged in the warp's shared memory as
// [y][x][z][c] (z contiguous, row stride padded so that the r row groups hit
// different banks).

constexpr int kBwdWarps = 4;

template <int C>
struct BwdSmem {
    static constexpr int kCol = 8 * C;              // floats per (y, x) column
    static constexpr int kRow = 8 * kCol + 4;       // floats per y row (+pad)
    static constexpr int kWarp = 8 * kRow;          // floats per warp buffer
};

// Stages dL/dvol of one tile, multiplied by 2^K with K chosen from the
// tile's largest |dL/dvol| so that the largest staged value lies in
// [2^64, 2^65) (K <= 126); returns K, or INT_MIN when the tile's gradient is
// zero (the tile contributes nothing). LOSS: dL/dvol is not materialised; it
// is the fused L1 gradient sign(vol - target) * scale, computed from the
// volume (passed as `grad`) and the target here.
template <int C, bool LOSS>
__device__ __forceinline__ int stage_grad_tile(const Geom &g,
                                                const float *__restrict__ grad,
                                                const float *__restrict__ target,
                                                float scale, int ox, int oy,
                                                int oz, float *buf, int lane) {
    using S = BwdSmem<C>;
    // 64 (z, y) rows of 8*C floats; lane handles rows lane and lane + 32
    float v[2][8 * C];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        const int row = lane + 32 * h;
        const int z = oz + (row >> 3), y = oy + (row & 7);
        const bool row_in = (z < g.z_end()) && (y < g.Y);
        const int nx = row_in ? min(kTile, g.X - ox) : 0;
        const size_t base =
            row_in ? (((size_t)(z - g.z_begin()) * g.Y + y) * g.X + ox) * C : 0;
        if (nx == kTile && (base & 3) == 0 &&
            ((reinterpret_cast<uintptr_t>(grad) & 15) == 0) &&
            (!LOSS || (reinterpret_cast<uintptr_t>(target) & 15) == 0)) {
#pragma unroll
            for (int q = 0; q < 2 * C; ++q) {
                const float4 t =
                    __ldg(reinterpret_cast<const float4 *>(grad + base) + q);
                v[h][4 * q + 0] = t.x;
                v[h][4 * q + 1] = t.y;
                v[h][4 * q + 2] = t.z;
                v[h][4 * q + 3] = t.w;
                if (LOSS) {
                    const float4 u =
                        __ldg(reinterpret_cast<const float4 *>(target + base) + q);
                    v[h][4 * q + 0] -= u.x;
                    v[h][4 * q + 1] -= u.y;
                    v[h][4 * q + 2] -= u.z;
                    v[h][4 * q + 3] -= u.w;
                }
            }
        } else {
#pragma unroll
            for (int q = 0; q < 8 * C; ++q) {
                v[h][q] = (q < nx * C) ? __ldg(grad + base + q) : 0.f;
                if (LOSS) v[h][q] -= (q < nx * C) ? __ldg(target + base + q) : 0.f;
            }
        }
        if (LOSS) {
#pragma unroll
            for (int q = 0; q < 8 * C; ++q)
                v[h][q] = v[h][q] > 0.f ? scale : (v[h][q] < 0.f ? -scale : 0.f);
        }
    }
    float m = 0.f;
    bool nan = false;
#pragma unroll
    for (int h = 0; h < 2; ++h)
#pragma unroll
        for (int q = 0; q < 8 * C; ++q) {
            m = fmaxf(m, fabsf(v[h][q]));
            nan |= v[h][q] != v[h][q];
        }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1)
        m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    // NaNs propagate as in the reference (staged unscaled in magnitude terms)
    if (__any_sync(0xffffffffu, nan)) m = fmaxf(m, 1.f);
    if (!(m > 0.f)) return INT_MIN;
    const int e = (int)((__float_as_uint(m) >> 23) & 0xff) - 127;
    const int K = min(126, 64 - e);
    const float gk = __uint_as_float((unsigned)(127 + K) << 23);
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        const int row = lane + 32 * h;
        const int zl = row >> 3, yl = row & 7;
#pragma unroll
        for (int x = 0; x < 8; ++x)
#pragma unroll
            for (int c = 0; c < C; ++c)
                buf[yl * S::kRow + x * S::kCol + c * 8 + zl] =
                    v[h][x * C + c] * gk;
    }
    return K;
}

// Sums over one y-row of the tile for one Gaussian (per lane).
struct RowSums {
    float R0, R1, R2, Rx0, Rxx, Rx1;
};

__device__ __forceinline__ float pick(const float2 (&p)[4], int j) {
    return (j & 1) ? p[j >> 1].y : p[j >> 1].x;
}

// Exact path: alpha = 2^s, counted where s >= thr (and s <= 0 unless the
// Gaussian is robustly positive definite), as the reference culls.
template <int C, bool CHECK_SIGN>
__device__ __forceinline__ RowSums bwd_row(const float *colbase, float mx,
                                           float thr, float A, float Cz,
                                           float E, float Dy, float By2,
                                           float Fy, const float2 (&dzp)[4],
                                           const float2 (&dsp)[4],
                                           const float (&I)[C],
                                           float (&W)[C]) {
    using S = BwdSmem<C>;
    RowSums r = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int x = 0; x < 8; ++x) {
        const float dx = mx - ((float)x + 0.5f);
        const float P = fmaf(dx, fmaf(A, dx, Dy), By2);
        const float L = fmaf(E, dx, Fy);
        float gv[8 * C];
#pragma unroll
        for (int q4 = 0; q4 < 2 * C; ++q4) {
            const float4 t =
                reinterpret_cast<const float4 *>(colbase + x * S::kCol)[q4];
            gv[4 * q4 + 0] = t.x;
            gv[4 * q4 + 1] = t.y;
            gv[4 * q4 + 2] = t.z;
            gv[4 * q4 + 3] = t.w;
        }
        float T0 = 0.f, T1 = 0.f, T2 = 0.f;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const float dzj = pick(dzp, j), dsj = pick(dsp, j);
            const float s = fmaf(dzj, fmaf(Cz, dzj, L), P);
            if (C == 1) {
                // w = alpha * dL/dvol; the three moment updates are
                // predicated on the cull test (no select instruction)
                const float w = ex2(s) * gv[j];
                if (CHECK_SIGN) {
                    asm("{\n\t.reg .pred p;\n\t"
                        "setp.ge.f32 p, %3, %4;\n\t"
                        "setp.le.and.f32 p, %3, 0f00000000, p;\n\t"
                        "@p add.f32 %0, %0, %5;\n\t"
                        "@p fma.rn.f32 %1, %5, %6, %1;\n\t"
                        "@p fma.rn.f32 %2, %5, %7, %2;\n\t}"
                        : "+f"(T0), "+f"(T1), "+f"(T2)
                        : "f"(s), "f"(thr), "f"(w), "f"(dzj), "f"(dsj));
                } else {
                    asm("{\n\t.reg .pred p;\n\t"
                        "setp.ge.f32 p, %3, %4;\n\t"
                        "@p add.f32 %0, %0, %5;\n\t"
                        "@p fma.rn.f32 %1, %5, %6, %1;\n\t"
                        "@p fma.rn.f32 %2, %5, %7, %2;\n\t}"
                        : "+f"(T0), "+f"(T1), "+f"(T2)
                        : "f"(s), "f"(thr), "f"(w), "f"(dzj), "f"(dsj));
                }
                continue;
            }
            bool ok = s >= thr;
            if (CHECK_SIGN) ok &= s <= 0.f;
            const float a = ok ? ex2(s) : 0.f;
            float w;
            {
                float h = I[0] * gv[j];
#pragma unroll
                for (int c = 1; c < C; ++c) h = fmaf(I[c], gv[c * 8 + j], h);
#pragma unroll
                for (int c = 0; c < C; ++c)
                    W[c] = fmaf(a, gv[c * 8 + j], W[c]);
                w = a * h;
            }
            T0 += w;
            T1 = fmaf(w, dzj, T1);
            T2 = fmaf(w, dsj, T2);
        }
        r.R0 += T0;
        r.R1 += T1;
        r.R2 += T2;
        const float u = dx * T0;
        r.Rx0 += u;
        r.Rxx = fmaf(u, dx, r.Rxx);
        r.Rx1 = fmaf(dx, T1, r.Rx1);
    }
    return r;
}

// Flush path (robustly positive-definite Gaussians): the row constant By2s
// carries -(thr + 126), so alpha' = 2^(s - thr - 126) is below the smallest
// normal float exactly when s < thr and ex2.approx.ftz returns 0 there: the
// cull costs no instruction. alpha = alpha' * 2^(thr + 126) is restored on
// the lane's sums. C = 1: two z-voxels per paired FP32 instruction
// (FFMA2 / FMUL2 / FADD2), sums kept as pairs until the end of the row.
__device__ __forceinline__ RowSums bwd_row_flush1(const float *colbase,
                                                  float mx, float A, float Cz,
                                                  float E, float Dy,
                                                  float By2s, float Fy,
                                                  const float2 (&dzp)[4],
                                                  const float2 (&dsp)[4]) {
    using S = BwdSmem<1>;
    const float2 z2 = f2(0.f), Cz2 = f2(Cz);
    float2 R0 = z2, R1 = z2, R2 = z2, Rx0 = z2, Rxx = z2, Rx1 = z2;
#pragma unroll
    for (int x = 0; x < 8; ++x) {
        const float dx = mx - ((float)x + 0.5f);
        const float2 dx2 = f2(dx);
        const float2 P = f2(fmaf(dx, fmaf(A, dx, Dy), By2s));
        const float2 L = f2(fmaf(E, dx, Fy));
        const float4 ga = reinterpret_cast<const float4 *>(colbase + x * S::kCol)[0];
        const float4 gb = reinterpret_cast<const float4 *>(colbase + x * S::kCol)[1];
        const float2 g[4] = {make_float2(ga.x, ga.y), make_float2(ga.z, ga.w),
                             make_float2(gb.x, gb.y), make_float2(gb.z, gb.w)};
        float2 T0, T1, T2;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const float2 sp = __ffma2_rn(dzp[k], __ffma2_rn(Cz2, dzp[k], L), P);
            const float2 w = __fmul2_rn(make_float2(ex2(sp.x), ex2(sp.y)), g[k]);
            if (k == 0) {
                T0 = w;
                T1 = __fmul2_rn(w, dzp[0]);
                T2 = __fmul2_rn(w, dsp[0]);
            } else {
                T0 = __fadd2_rn(T0, w);
                T1 = __ffma2_rn(w, dzp[k], T1);
                T2 = __ffma2_rn(w, dsp[k], T2);
            }
        }
        R0 = __fadd2_rn(R0, T0);
        R1 = __fadd2_rn(R1, T1);
        R2 = __fadd2_rn(R2, T2);
        const float2 u = __fmul2_rn(dx2, T0);
        Rx0 = __fadd2_rn(Rx0, u);
        Rxx = __ffma2_rn(u, dx2, Rxx);
        Rx1 = __ffma2_rn(dx2, T1, Rx1);
    }
    RowSums r;
    r.R0 = R0.x + R0.y;
    r.R1 = R1.x + R1.y;
    r.R2 = R2.x + R2.y;
    r.Rx0 = Rx0.x + Rx0.y;
    r.Rxx = Rxx.x + Rxx.y;
    r.Rx1 = Rx1.x + Rx1.y;
    return r;
}

// Flush path for C > 1: as bwd_row_flush1, two z-voxels per paired
// instruction; h = sum_c I_c dL/dvol_c and the channel sums W_c are kept as
// (even z, odd z) pairs, collapsed by the caller.
template <int C>
__device__ __forceinline__ RowSums bwd_row_flushc(const float *colbase,
                                                  float mx, float A, float Cz,
                                                  float E, float Dy, float By2s,
                                                  float Fy,
                                                  const float2 (&dzp)[4],
                                                  const float2 (&dsp)[4],
                                                  const float (&I)[C],
                                                  float2 (&W2)[C]) {
    using S = BwdSmem<C>;
    const float2 z2 = f2(0.f), Cz2 = f2(Cz);
    float2 R0 = z2, R1 = z2, R2 = z2, Rx0 = z2, Rxx = z2, Rx1 = z2;
#pragma unroll
    for (int x = 0; x < 8; ++x) {
        const float dx = mx - ((float)x + 0.5f);
        const float2 dx2 = f2(dx);
        const float2 P = f2(fmaf(dx, fmaf(A, dx, Dy), By2s));
        const float2 L = f2(fmaf(E, dx, Fy));
        // dL/dvol of column x, [c][z]: 4 pairs per channel
        float2 g[C][4];
#pragma unroll
        for (int c = 0; c < C; ++c) {
            const float4 ga =
                reinterpret_cast<const float4 *>(colbase + x * S::kCol + c * 8)[0];
            const float4 gb =
                reinterpret_cast<const float4 *>(colbase + x * S::kCol + c * 8)[1];
            g[c][0] = make_float2(ga.x, ga.y);
            g[c][1] = make_float2(ga.z, ga.w);
            g[c][2] = make_float2(gb.x, gb.y);
            g[c][3] = make_float2(gb.z, gb.w);
        }
        float2 T0, T1, T2;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const float2 sp = __ffma2_rn(dzp[k], __ffma2_rn(Cz2, dzp[k], L), P);
            const float2 a = make_float2(ex2(sp.x), ex2(sp.y));
            float2 h = __fmul2_rn(f2(I[0]), g[0][k]);
#pragma unroll
            for (int c = 1; c < C; ++c) h = __ffma2_rn(f2(I[c]), g[c][k], h);
#pragma unroll
            for (int c = 0; c < C; ++c) W2[c] = __ffma2_rn(a, g[c][k], W2[c]);
            const float2 w = __fmul2_rn(a, h);
            if (k == 0) {
                T0 = w;
                T1 = __fmul2_rn(w, dzp[0]);
                T2 = __fmul2_rn(w, dsp[0]);
            } else {
                T0 = __fadd2_rn(T0, w);
                T1 = __ffma2_rn(w, dzp[k], T1);
                T2 = __ffma2_rn(w, dsp[k], T2);
            }
        }
        R0 = __fadd2_rn(R0, T0);
        R1 = __fadd2_rn(R1, T1);
        R2 = __fadd2_rn(R2, T2);
        const float2 u = __fmul2_rn(dx2, T0);
        Rx0 = __fadd2_rn(Rx0, u);
        Rxx = __ffma2_rn(u, dx2, Rxx);
        Rx1 = __ffma2_rn(dx2, T1, Rx1);
    }
    RowSums r;
    r.R0 = R0.x + R0.y;
    r.R1 = R1.x + R1.y;
    r.R2 = R2.x + R2.y;
    r.Rx0 = Rx0.x + Rx0.y;
    r.Rxx = Rxx.x + Rxx.y;
    r.Rx1 = Rx1.x + Rx1.y;
    return r;
}

// Lanes of a work item of m Gaussians: r row groups of gs = 32 / r lanes
// (r the largest power of two <= 8 with m * r <= 32); lane = sub * gs + gi
// evaluates Gaussian slot gi over the tile's y-rows [sub * rows, +rows).
struct ItemLanes {
    int gs, gi, sub, rows;
    bool valid;
};

__device__ __forceinline__ ItemLanes item_lanes(int m, int lane) {
    int r = 1;
    while (r < 8 && m * r * 2 <= 32) r <<= 1;
    ItemLanes L;
    L.gs = 32 / r;
    L.gi = lane & (L.gs - 1);
    L.sub = lane >> (__ffs(L.gs) - 1);
    L.rows = 8 / r;
    L.valid = L.gi < m;
    return L;
}

// One work item's evaluation, from the staged (2^K-scaled) dL/dvol tile in
// `buf` and the lane's record (r0 tile-relative; invalid lanes: thr NaN),
// to the per-Gaussian atomics.
template <int C>
__device__ __forceinline__ void bwd_item(const float *buf, int K,
                                         const ItemLanes &L, int gid,
                                         const float4 &r0, const float4 &r1,
                                         const float4 &r2, const float4 &r3,
                                         float *__restrict__ pos_grad,
                                         float *__restrict__ conic_grad,
                                         float *__restrict__ int_grad) {
    using S = BwdSmem<C>;
    float I[C];
    record_intensity<C>(r2, r3, I);
    const float thr = r0.w;
    const bool all_robust = __all_sync(0xffffffffu, robust_flag(thr));
    // flush path: every valid lane robust with thr >= -126, and the tile's
    // scale leaves 2^(thr + 126 - K) finite (K >= -1)
    const bool flush =
        K >= -1 && __all_sync(0xffffffffu,
                              !L.valid || (robust_flag(thr) && thr >= -126.f));
    const float shift = L.valid ? thr + 126.f : __int_as_float(0x7f800000);
    float2 dzp[4], dsp[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        dzp[k] = make_float2(r0.z - ((float)(2 * k) + 0.5f),
                             r0.z - ((float)(2 * k + 1) + 0.5f));
        dsp[k] = __fmul2_rn(dzp[k], dzp[k]);
    }

    // sums over the Gaussian's voxels of w-weighted monomials of d, where
    // w = alpha * h and h = sum_c I_c dL/dvol_c (C > 1) or dL/dvol (C = 1)
    float Sxx = 0.f, Syy = 0.f, Szz = 0.f, Sxy = 0.f, Sxz = 0.f, Syz = 0.f;
    float Vx = 0.f, Vy = 0.f, Vz = 0.f;
    float W[C];
    float2 W2[C];  // flush path, C > 1: (even z, odd z) channel sums
#pragma unroll
    for (int c = 0; c < C; ++c) {
        W[c] = 0.f;
        W2[c] = make_float2(0.f, 0.f);
    }

#pragma unroll 1
    for (int q = 0; q < L.rows; ++q) {
        const int yl = L.sub * L.rows + q;
        const float dy = r0.y - ((float)yl + 0.5f);
        const float By2 = r1.y * dy * dy, Dy = r1.w * dy, Fy = r2.y * dy;
        const float *colbase = buf + yl * S::kRow;
        RowSums rs;
        if (flush) {
            if (C == 1)
                rs = bwd_row_flush1(colbase, r0.x, r1.x, r1.z, r2.x, Dy,
                                    By2 - shift, Fy, dzp, dsp);
            else
                rs = bwd_row_flushc<C>(colbase, r0.x, r1.x, r1.z, r2.x, Dy,
                                       By2 - shift, Fy, dzp, dsp, I, W2);
        } else if (all_robust) {
            rs = bwd_row<C, false>(colbase, r0.x, thr, r1.x, r1.z, r2.x, Dy,
                                   By2, Fy, dzp, dsp, I, W);
        } else {
            rs = bwd_row<C, true>(colbase, r0.x, thr, r1.x, r1.z, r2.x, Dy,
                                  By2, Fy, dzp, dsp, I, W);
        }
        if (C == 1) W[0] += rs.R0;  // intensity grad = sum(w) (C = 1)
        Sxx += rs.Rxx;
        Szz += rs.R2;
        Sxz += rs.Rx1;
        Vx += rs.Rx0;
        Vz += rs.R1;
        Syy = fmaf(dy * dy, rs.R0, Syy);
        Sxy = fmaf(dy, rs.Rx0, Sxy);
        Syz = fmaf(dy, rs.R1, Syz);
        Vy = fmaf(dy, rs.R0, Vy);
    }

    if (C > 1) {
#pragma unroll
        for (int c = 0; c < C; ++c) W[c] += W2[c].x + W2[c].y;
    }

    // combine row groups (lanes gi, gi+gs, gi+2gs, ...)
    for (int o = L.gs; o < 32; o <<= 1) {
        Sxx += __shfl_xor_sync(0xffffffffu, Sxx, o);
        Syy += __shfl_xor_sync(0xffffffffu, Syy, o);
        Szz += __shfl_xor_sync(0xffffffffu, Szz, o);
        Sxy += __shfl_xor_sync(0xffffffffu, Sxy, o);
        Sxz += __shfl_xor_sync(0xffffffffu, Sxz, o);
        Syz += __shfl_xor_sync(0xffffffffu, Syz, o);
        Vx += __shfl_xor_sync(0xffffffffu, Vx, o);
        Vy += __shfl_xor_sync(0xffffffffu, Vy, o);
        Vz += __shfl_xor_sync(0xffffffffu, Vz, o);
#pragma unroll
        for (int c = 0; c < C; ++c) W[c] += __shfl_xor_sync(0xffffffffu, W[c], o);
    }

    if (L.valid && L.sub == 0) {
        // undo the staging scale 2^K and, on the flush path, the exponent
        // shift 2^-(thr + 126)
        const float corr = flush ? ex2(fminf(shift - (float)K, 127.f))
                                 : __uint_as_float((unsigned)(127 - K) << 23);
#pragma unroll
        for (int c = 0; c < C; ++c) W[c] *= corr;
        const float k = ((C == 1) ? I[0] : 1.f) * corr;  // sigma_grad = I * w
        // -Q (conic) from the record: r1 = (h a, h d, h f, -log2e b),
        // r2 = (-log2e c, -log2e e, ..) with h = -log2e / 2
        const float nqa = 2.f * kLn2 * r1.x, nqd = 2.f * kLn2 * r1.y,
                    nqf = 2.f * kLn2 * r1.z, nqb = kLn2 * r1.w,
                    nqc = kLn2 * r2.x, nqe = kLn2 * r2.y;
        const float vx = k * Vx, vy = k * Vy, vz = k * Vz;
        red_add4(pos_grad + 4 * (size_t)gid, nqa * vx + nqb * vy + nqc * vz,
                 nqb * vx + nqd * vy + nqe * vz, nqc * vx + nqe * vy + nqf * vz,
                 0.f);
        float *cg = conic_grad + 6 * (size_t)gid;
        red_add2(cg + 0, -0.5f * k * Sxx, -k * Sxy);
        red_add2(cg + 2, -k * Sxz, -0.5f * k * Syy);
        red_add2(cg + 4, -k * Syz, -0.5f * k * Szz);
        float *ig = int_grad + (size_t)C * gid;
        if (C == 4) {
            red_add4(ig, W[0], W[C > 1 ? 1 : 0], W[C > 2 ? 2 : 0],
                     W[C > 3 ? 3 : 0]);
        } else if (C == 2) {
            red_add2(ig, W[0], W[C > 1 ? 1 : 0]);
        } else {
#pragma unroll
            for (int c = 0; c < C; ++c) red_add(ig + c, W[c]);
        }
    }
}

// Record of an item's lane: loaded, made tile-relative; invalid lanes get
// thr = NaN (nothing passes) and zero coefficients.
template <int R>
__device__ __forceinline__ void item_record(const float4 *__restrict__ rec,
                                            int gid, bool valid, int ox,
                                            int oy, int oz, float4 &r0,
                                            float4 &r1, float4 &r2,
                                            float4 &r3) {
    r0 = make_float4(0.f, 0.f, 0.f, __int_as_float(0x7f800001));
    r1 = make_float4(0.f, 0.f, 0.f, 0.f);
    r2 = r1;
    r3 = r1;
    if (valid) {
        r0 = rec[(size_t)gid * R + 0];
        r1 = rec[(size_t)gid * R + 1];
        r2 = rec[(size_t)gid * R + 2];
        if (R == 4) r3 = rec[(size_t)gid * R + 3];
        r0.x -= (float)ox;
        r0.y -= (float)oy;
        r0.z -= (float)oz;
    }
}

// Per-Gaussian backward: persistent warps take items from an atomic
// counter; each item stages its tile, loads its records and evaluates.
template <int C, bool LOSS>
__global__ void __launch_bounds__(kBwdWarps * 32, C <= 2 ? 5 : 4)
vox_bwd_gauss_kernel(Geom g, const int *__restrict__ ids,
                     const float4 *__restrict__ rec,
                     const float2 *__restrict__ conics,
                     const float *__restrict__ grad,
                     const int4 *__restrict__ item_desc,
                     const long long *__restrict__ item_total,
                     int *__restrict__ work_counter,
                     float *__restrict__ pos_grad,
                     float *__restrict__ conic_grad,
                     float *__restrict__ int_grad,
                     const float *__restrict__ target,
                     const float *__restrict__ grad_loss, float inv_denom) {
    using S = BwdSmem<C>;
    constexpr int R = Rec<C>::kF4;
    __shared__ __align__(16) float smem[kBwdWarps * S::kWarp];
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    float *buf = smem + wid * S::kWarp;
    const int total = (int)*item_total;
    const float scale = LOSS ? (*grad_loss) * inv_denom : 0.f;

    while (true) {
        int item = 0;
        if (lane == 0) item = atomicAdd(work_counter, 1);
        item = __shfl_sync(0xffffffffu, item, 0);
        if (item >= total) break;
        const int4 d = __ldg(item_desc + item);
        const ItemLanes L = item_lanes(d.z, lane);
        int ox, oy, oz;
        tile_coords(g, d.x, ox, oy, oz);
        // records first: their loads are in flight while the tile stages
        const int gid = L.valid ? __ldg(ids + d.y + L.gi) : 0;
        float4 r0, r1, r2, r3;
        item_record<R>(rec, gid, L.valid, ox, oy, oz, r0, r1, r2, r3);
        __syncwarp();
        const int K = stage_grad_tile<C, LOSS>(g, grad, target, scale, ox, oy,
                                               oz, buf, lane);
        __syncwarp();
        if (K == INT_MIN) continue;  // dL/dvol is zero on this tile
        bwd_item<C>(buf, K, L, gid, r0, r1, r2, r3, pos_grad, conic_grad,
                    int_grad);
    }
}

// Per-tile item counts (ceil(n_t / 32)) for the planner.
__global__ void __launch_bounds__(256)
item_count_kernel(const int2 *__restrict__ bins, long long ntiles,
                  int *__restrict__ counts) {
    const long long t = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= ntiles) return;
    const int2 r = bins[t];
    const int n = max(0, r.y - r.x);
    counts[t] = (n + 31) / 32;
}

// Item descriptors (tile, first pair, number of Gaussians <= 32, 0).
__global__ void __launch_bounds__(256)
item_fill_kernel(const int2 *__restrict__ bins,
                 const int2 *__restrict__ item_bins, long long ntiles,
                 int4 *__restrict__ item_desc) {
    const long long t = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= ntiles) return;
    const int2 r = item_bins[t];
    const int2 range = bins[t];
    for (int k = r.x; k < r.y; ++k) {
        const int start = range.x + 32 * (k - r.x);
        item_desc[k] = make_int4((int)t, start, min(32, range.y - start), 0);
    }
}

// ------------------------------------------------------ backward (per voxel)
//
// Voxel-centric variant (the reference's use_per_gaussian_backward=False):
// one CTA of 64 threads per tile, one thread per (x, y) column of 8 voxels;
// each thread folds its column into the per-Gaussian sums, the warp reduces
// them, and lane 0 issues one set of vector atomics per warp and Gaussian.

constexpr int kVoxThreads = 64;
constexpr int kVoxBatch = 128;

template <int C>
__global__ void __launch_bounds__(kVoxThreads, C <= 2 ? 16 : 8)
vox_bwd_voxel_kernel(Geom g, const int2 *__restrict__ bins,
                     const int *__restrict__ ids,
                     const float4 *__restrict__ rec,
                     const float2 *__restrict__ conics,
                     const float *__restrict__ grad,
                     float *__restrict__ pos_grad,
                     float *__restrict__ conic_grad,
                     float *__restrict__ int_grad) {
    constexpr int R = Rec<C>::kF4;
    __shared__ __align__(16) float4 sb[kVoxBatch * R];
    __shared__ int sid[kVoxBatch];

    const long long tile = blockIdx.x;
    int ox, oy, oz;
    tile_coords(g, tile, ox, oy, oz);
    const int lane = threadIdx.x & 31;
    const int lx = threadIdx.x & 7, ly = threadIdx.x >> 3;
    const float fx = lx + 0.5f, fy = ly + 0.5f;

    // this thread's column of dL/dvol (zero outside the volume)
    float gv[8][C];
    {
        const int x = ox + lx, y = oy + ly;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const int z = oz + j;
            const bool in = x < g.X && y < g.Y && z < g.z_end();
            const size_t base =
                in ? (((size_t)(z - g.z_begin()) * g.Y + y) * g.X + x) * C : 0;
#pragma unroll
            for (int c = 0; c < C; ++c) gv[j][c] = in ? grad[base + c] : 0.f;
        }
    }

    const int2 range = bins[tile];
    for (int s0 = range.x; s0 < range.y; s0 += kVoxBatch) {
        const int nb = min(kVoxBatch, range.y - s0);
        __syncthreads();
        for (int k = threadIdx.x; k < nb; k += kVoxThreads) {
            const int gid = ids[s0 + k];
            sid[k] = gid;
            float4 r0 = rec[(size_t)gid * R];
            r0.x -= (float)ox;
            r0.y -= (float)oy;
            r0.z -= (float)oz;
            sb[k * R] = r0;
#pragma unroll
            for (int q = 1; q < R; ++q) sb[k * R + q] = rec[(size_t)gid * R + q];
        }
        __syncthreads();
#pragma unroll 1
        for (int t = 0; t < nb; ++t) {
            const float4 r0 = sb[t * R + 0];
            const float4 r1 = sb[t * R + 1];
            const float4 r2 = sb[t * R + 2];
            const float4 r3 = (R == 4) ? sb[t * R + 3] : r2;
            float I[C];
            record_intensity<C>(r2, r3, I);
            const float dx = r0.x - fx, dy = r0.y - fy;
            const float P = fmaf(dx, fmaf(r1.x, dx, r1.w * dy), r1.y * dy * dy);
            const float L = fmaf(r2.x, dx, r2.y * dy);
            const float thr = r0.w;
            const bool check_sign = !robust_flag(thr);
            float T0 = 0.f, T1 = 0.f, T2 = 0.f;
            float W[C];
#pragma unroll
            for (int c = 0; c < C; ++c) W[c] = 0.f;
            bool touched = false;
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const float dz = r0.z - ((float)j + 0.5f);
                const float s = fmaf(dz, fmaf(r1.z, dz, L), P);
                const bool ok = (s >= thr) & (!check_sign | (s <= 0.f));
                const float a = ok ? ex2(s) : 0.f;
                float h = I[0] * gv[j][0];
#pragma unroll
                for (int c = 1; c < C; ++c) h = fmaf(I[c], gv[j][c], h);
#pragma unroll
                for (int c = 0; c < C; ++c) W[c] = fmaf(a, gv[j][c], W[c]);
                const float w = a * h;
                touched |= (a != 0.f);
                T0 += w;
                const float tt = w * dz;
                T1 += tt;
                T2 = fmaf(tt, dz, T2);
            }
            if (!__any_sync(0xffffffffu, touched)) continue;
            float v[9 + C];
            v[0] = dx * dx * T0;  // Sxx
            v[1] = dy * dy * T0;  // Syy
            v[2] = T2;            // Szz
            v[3] = dx * dy * T0;  // Sxy
            v[4] = dx * T1;       // Sxz
            v[5] = dy * T1;       // Syz
            v[6] = dx * T0;       // Vx
            v[7] = dy * T0;       // Vy
            v[8] = T1;            // Vz
#pragma unroll
            for (int c = 0; c < C; ++c) v[9 + c] = W[c];
#pragma unroll
            for (int k = 0; k < 9 + C; ++k)
#pragma unroll
                for (int o = 16; o > 0; o >>= 1)
                    v[k] += __shfl_xor_sync(0xffffffffu, v[k], o);
            if (lane == 0) {
                const int gid = sid[t];
                const float2 ab = conics[3 * gid + 0],
                             cd = conics[3 * gid + 1],
                             ef = conics[3 * gid + 2];
                red_add4(pos_grad + 4 * (size_t)gid,
                         -(ab.x * v[6] + ab.y * v[7] + cd.x * v[8]),
                         -(ab.y * v[6] + cd.y * v[7] + ef.x * v[8]),
                         -(cd.x * v[6] + ef.x * v[7] + ef.y * v[8]), 0.f);
                float *cg = conic_grad + 6 * (size_t)gid;
                red_add2(cg + 0, -0.5f * v[0], -v[3]);
                red_add2(cg + 2, -v[4], -0.5f * v[1]);
                red_add2(cg + 4, -v[5], -0.5f * v[2]);
                float *ig = int_grad + (size_t)C * gid;
#pragma unroll
                for (int c = 0; c < C; ++c) red_add(ig + c, v[9 + c]);
            }
        }
    }
}

// Zeroes the three gradient arrays and the work counter in one launch.
__global__ void __launch_bounds__(256)
zero_grads_kernel(int n, int C, float *__restrict__ pos_grad,
                  float *__restrict__ conic_grad, float *__restrict__ int_grad,
                  int *__restrict__ counter) {
    const long long tid = (long long)blockIdx.x * blockDim.x + threadIdx.x;
    const long long stride = (long long)gridDim.x * blockDim.x;
    if (tid < 4) counter[tid] = 0;
    for (long long i = tid; i < n; i += stride) {
        reinterpret_cast<float4 *>(pos_grad)[i] = make_float4(0.f, 0.f, 0.f, 0.f);
        reinterpret_cast<float2 *>(conic_grad)[3 * i + 0] = make_float2(0.f, 0.f);
        reinterpret_cast<float2 *>(conic_grad)[3 * i + 1] = make_float2(0.f, 0.f);
        reinterpret_cast<float2 *>(conic_grad)[3 * i + 2] = make_float2(0.f, 0.f);
        for (int c = 0; c < C; ++c) int_grad[i * C + c] = 0.f;
    }
}

}  // namespace

// ------------------------------------------------------------ host launchers

struct VoxLayout {
    size_t rec, item_counts, item_bins, partials, item_desc, counter,
        tile_loss, loss_partials, total;
};

static inline size_t align256v(size_t x) { return (x + 255) & ~size_t(255); }

VoxLayout vox_layout(long long n, int channels, long long ntiles,
                     long long nisect) {
    VoxLayout L;
    const int R = channels <= 2 ? 3 : 4;
    const long long nblocks = scan_blocks(ntiles);
    const long long max_items = (nisect + 31) / 32 + ntiles;
    size_t off = 0;
    L.rec = off;
    off = align256v(off + sizeof(float4) * (size_t)R * (size_t)(n > 0 ? n : 1));
    L.item_counts = off;
    off = align256v(off + sizeof(int) * (size_t)ntiles);
    L.item_bins = off;
    off = align256v(off + sizeof(int2) * (size_t)ntiles);
    L.partials = off;
    off = align256v(off + sizeof(long long) * (size_t)(nblocks + 1));
    L.item_desc = off;
    off = align256v(off + sizeof(int4) * (size_t)(max_items + 1));
    L.counter = off;
    off = align256v(off + sizeof(int) * 4);
    L.tile_loss = off;
    off = align256v(off + sizeof(float) * (size_t)(ntiles > 0 ? ntiles : 1));
    L.loss_partials = off;  // sized for any reduction (<= kSMs*8 blocks)
    off = align256v(off + l1_workspace_bytes(1LL << 40));
    L.total = off;
    return L;
}

size_t vox_workspace_bytes(long long n, int channels, long long ntiles,
                           long long nisect) {
    return vox_layout(n, channels, ntiles, nisect).total;
}

static cudaError_t launch_prep(int n, int C, const float *pos_radii,
                               const float *conics, const float *intens,
                               float4 *rec, cudaStream_t stream) {
    if (n <= 0) return cudaSuccess;
    const int blocks = (n + 255) / 256;
    const float4 *p = reinterpret_cast<const float4 *>(pos_radii);
    const float2 *q = reinterpret_cast<const float2 *>(conics);
    switch (C) {
        case 1: prep_records_kernel<1><<<blocks, 256, 0, stream>>>(n, p, q, intens, rec); break;
        case 2: prep_records_kernel<2><<<blocks, 256, 0, stream>>>(n, p, q, intens, rec); break;
        case 3: prep_records_kernel<3><<<blocks, 256, 0, stream>>>(n, p, q, intens, rec); break;
        case 4: prep_records_kernel<4><<<blocks, 256, 0, stream>>>(n, p, q, intens, rec); break;
        default: return cudaErrorInvalidValue;
    }
    count_launches(1);
    return cudaGetLastError();
}

template <int C, bool LOSS>
static void fwd_launch(unsigned grid, cudaStream_t stream, const Geom &g,
                       const int2 *bins, const int *ids, const float4 *rec,
                       float *out, const float *target, float *tile_loss,
                       float *sign_plane = nullptr, int *tile_of = nullptr) {
    vox_fwd_kernel<C, LOSS><<<grid, 32, 0, stream>>>(
        g, bins, ids, rec, out, target, tile_loss, sign_plane, tile_of);
}

// target != nullptr: fused L1, loss_out[0] = sum |vol - target| * inv_denom;
// sign_plane / tile_of (C = 1, fused L1, optional): the inputs of the
// tensor-core backward (bwd_tc.cu)
cudaError_t launch_vox_forward_ex(const Geom &g, int C, int n, long long nisect,
                               const int *ids,
                               const int *tile_bins, const float *pos_radii,
                               const float *conics, const float *intens,
                               float *out, void *ws, cudaStream_t stream,
                               const float *target, float *loss_out,
                               double inv_denom, float *sign_plane,
                               int *tile_of) {
    const long long ntiles = g.slab_tiles();
    // the same layout as the backward's: the fused-L1 forward's binning has
    // already written the backward's work plan into this workspace
    const VoxLayout L = vox_layout(n, C, ntiles, nisect);
    char *base = static_cast<char *>(ws);
    float4 *rec = reinterpret_cast<float4 *>(base + L.rec);
    float *tile_loss = reinterpret_cast<float *>(base + L.tile_loss);
    cudaError_t err = launch_prep(n, C, pos_radii, conics, intens, rec, stream);
    if (err) return err;
    if (ntiles == 0) {
        if (target) return cudaMemsetAsync(loss_out, 0, sizeof(float), stream);
        return cudaSuccess;
    }
    const int2 *bins = reinterpret_cast<const int2 *>(tile_bins);
    const unsigned grid = (unsigned)ntiles;
    profile_mark(kProfForward, false, stream);
    const bool loss = target != nullptr;
    switch (C * 2 + (loss ? 1 : 0)) {
        case 2: fwd_launch<1, false>(grid, stream, g, bins, ids, rec, out, target, tile_loss); break;
        case 3: fwd_launch<1, true>(grid, stream, g, bins, ids, rec, out, target, tile_loss,
                                    sign_plane, tile_of); break;
        case 4: fwd_launch<2, false>(grid, stream, g, bins, ids, rec, out, target, tile_loss); break;
        case 5: fwd_launch<2, true>(grid, stream, g, bins, ids, rec, out, target, tile_loss); break;
        case 6: fwd_launch<3, false>(grid, stream, g, bins, ids, rec, out, target, tile_loss); break;
        case 7: fwd_launch<3, true>(grid, stream, g, bins, ids, rec, out, target, tile_loss); break;
        case 8: fwd_launch<4, false>(grid, stream, g, bins, ids, rec, out, target, tile_loss); break;
        case 9: fwd_launch<4, true>(grid, stream, g, bins, ids, rec, out, target, tile_loss); break;
        default: return cudaErrorInvalidValue;
    }
    profile_mark(kProfForward, true, stream);
    count_launches(1);
    if ((err = cudaGetLastError())) return err;
    if (loss)
        return launch_sum(ntiles, tile_loss, nullptr, inv_denom, loss_out,
                          base + L.loss_partials, stream);
    return cudaSuccess;
}

cudaError_t launch_vox_forward(const Geom &g, int C, int n, long long nisect,
                               const int *ids, const int *tile_bins,
                               const float *pos_radii, const float *conics,
                               const float *intens, float *out, void *ws,
                               cudaStream_t stream, const float *target,
                               float *loss_out, double inv_denom) {
    return launch_vox_forward_ex(g, C, n, nisect, ids, tile_bins, pos_radii,
                                 conics, intens, out, ws, stream, target,
                                 loss_out, inv_denom, nullptr, nullptr);
}

// Fused-L1 forward of an empty tile list: the volume is zero, so the loss is
// sum |target| * inv_denom.
cudaError_t launch_empty_l1(long long nvox, const float *target,
                            double inv_denom, float *loss_out, void *ws,
                            cudaStream_t stream) {
    const VoxLayout L = vox_layout(0, 1, 0, 0);
    return launch_sum(nvox, target, nullptr, inv_denom, loss_out,
                      static_cast<char *>(ws) + L.loss_partials, stream);
}

template <int C, bool LOSS>
static int bwd_gauss_grid() {
    static int cached = 0;
    if (cached) return cached;
    int per_sm = 0;
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(
            &per_sm, vox_bwd_gauss_kernel<C, LOSS>, kBwdWarps * 32, 0);
    int dev = 0, sms = kSMs;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    cached = std::max(1, per_sm) * sms;
    return cached;
}

template <int C, bool LOSS>
static void bwd_launch(cudaStream_t stream, const Geom &g, const int *ids,
                       const float4 *rec, const float2 *cq, const float *grad,
                       const int4 *item_desc, const long long *total,
                       int *counter, float *pos_grad, float *conic_grad,
                       float *int_grad, const float *target,
                       const float *grad_loss, float inv_denom) {
    vox_bwd_gauss_kernel<C, LOSS><<<bwd_gauss_grid<C, LOSS>(), kBwdWarps * 32,
                                    0, stream>>>(
        g, ids, rec, cq, grad, item_desc, total, counter, pos_grad,
        conic_grad, int_grad, target, grad_loss, inv_denom);
}

// Backward work plan from tile_bins: per-tile bucket counts, their scan and
// the item descriptors (the kernel's work queue).
static cudaError_t launch_bwd_plan(const int2 *bins, long long ntiles,
                                   int *item_counts, long long *partials,
                                   int *item_bins, int4 *item_desc,
                                   cudaStream_t stream) {
    const unsigned tblocks = (unsigned)((ntiles + 255) / 256);
    item_count_kernel<<<tblocks, 256, 0, stream>>>(bins, ntiles, item_counts);
    cudaError_t err = scan_counts_to_bins(item_counts, ntiles, partials,
                                          item_bins, stream, LLONG_MAX);
    if (err) return err;
    item_fill_kernel<<<tblocks, 256, 0, stream>>>(
        bins, reinterpret_cast<const int2 *>(item_bins), ntiles, item_desc);
    count_launches(2);
    return cudaGetLastError();
}

// The work-plan buffers of the vox workspace, for the binning to fill
// (ItemScan) in the fused-L1 forward.
ItemScan vox_item_scan(void *ws, long long n, int C, long long ntiles,
                       long long nisect) {
    const VoxLayout L = vox_layout(n, C, ntiles, nisect);
    char *base = static_cast<char *>(ws);
    ItemScan it;
    it.partials = reinterpret_cast<long long *>(base + L.partials);
    it.item_bins = reinterpret_cast<int *>(base + L.item_bins);
    it.desc = reinterpret_cast<int4 *>(base + L.item_desc);
    it.cap = (nisect + 31) / 32 + ntiles;
    return it;
}

// target != nullptr: fused L1; `grad` is then the forward volume and
// dL/dvol = sign(vol - target) * grad_loss[0] * inv_denom.
cudaError_t launch_vox_backward_gauss(const Geom &g, int C, int n,
                                      long long nisect, const int *ids,
                                      const int *tile_bins,
                                      const float *pos_radii,
                                      const float *conics,
                                      const float *intens, const float *grad,
                                      float *pos_grad, float *conic_grad,
                                      float *int_grad, void *ws,
                                      cudaStream_t stream,
                                      const float *target,
                                      const float *grad_loss,
                                      float inv_denom, int stage,
                                      const TcInputs *tc) {
    const long long ntiles = g.slab_tiles();
    const VoxLayout L = vox_layout(n, C, ntiles, nisect);
    char *base = static_cast<char *>(ws);
    float4 *rec = reinterpret_cast<float4 *>(base + L.rec);
    int *item_counts = reinterpret_cast<int *>(base + L.item_counts);
    int *item_bins = reinterpret_cast<int *>(base + L.item_bins);
    long long *partials = reinterpret_cast<long long *>(base + L.partials);
    int4 *item_desc = reinterpret_cast<int4 *>(base + L.item_desc);
    int *counter = reinterpret_cast<int *>(base + L.counter);
    const long long nblocks = scan_blocks(ntiles);

    cudaError_t err;
    const int2 *bins = reinterpret_cast<const int2 *>(tile_bins);
    if (stage == kBwdPrepared) {
        zero_grads_kernel<<<std::max(1, std::min((n + 255) / 256, kSMs * 8)),
                            256, 0, stream>>>(n, C, pos_grad, conic_grad,
                                              int_grad, counter);
        count_launches(1);
        if ((err = cudaGetLastError())) return err;
        if (n <= 0 || ntiles == 0 || nisect <= 0) return cudaSuccess;
    } else {
        if ((err = cudaMemsetAsync(pos_grad, 0, sizeof(float) * 4 * (size_t)n, stream))) return err;
        if ((err = cudaMemsetAsync(conic_grad, 0, sizeof(float) * 6 * (size_t)n, stream))) return err;
        if ((err = cudaMemsetAsync(int_grad, 0, sizeof(float) * C * (size_t)n, stream))) return err;
        if (n <= 0 || ntiles == 0 || nisect <= 0) return cudaSuccess;
        if ((err = cudaMemsetAsync(counter, 0, sizeof(int) * 4, stream))) return err;
        if ((err = launch_prep(n, C, pos_radii, conics, intens, rec, stream))) return err;
        if ((err = launch_bwd_plan(bins, ntiles, item_counts, partials,
                                   item_bins, item_desc, stream)))
            return err;
    }
    const long long *total = partials + nblocks;
    const float2 *cq = reinterpret_cast<const float2 *>(conics);
    const bool loss = target != nullptr;
    if (stage == kBwdPrepared && tc && C == 1 && loss) {
        profile_mark(kProfBackwardGauss, false, stream);
        err = launch_vox_backward_tc(g, ids, tc->tile_of, rec, tc->sign_plane,
                                     tc->pair_total, nisect, pos_grad,
                                     conic_grad, int_grad, grad_loss,
                                     inv_denom, stream);
        profile_mark(kProfBackwardGauss, true, stream);
        return err;
    }
    profile_mark(kProfBackwardGauss, false, stream);
#define GSV_BWD(Cc, Ll)                                                       \
    bwd_launch<Cc, Ll>(stream, g, ids, rec, cq, grad, item_desc, total,       \
                       counter, pos_grad, conic_grad, int_grad, target,        \
                       grad_loss, inv_denom)
    switch (C * 2 + (loss ? 1 : 0)) {
        case 2: GSV_BWD(1, false); break;
        case 3: GSV_BWD(1, true); break;
        case 4: GSV_BWD(2, false); break;
        case 5: GSV_BWD(2, true); break;
        case 6: GSV_BWD(3, false); break;
        case 7: GSV_BWD(3, true); break;
        case 8: GSV_BWD(4, false); break;
        case 9: GSV_BWD(4, true); break;
        default: return cudaErrorInvalidValue;
    }
#undef GSV_BWD
    profile_mark(kProfBackwardGauss, true, stream);
    count_launches(1);
    return cudaGetLastError();
}

cudaError_t launch_vox_backward_voxel(const Geom &g, int C, int n,
                                      long long nisect, const int *ids,
                                      const int *tile_bins,
                                      const float *pos_radii,
                                      const float *conics,
                                      const float *intens, const float *grad,
                                      float *pos_grad, float *conic_grad,
                                      float *int_grad, void *ws,
                                      cudaStream_t stream) {
    const long long ntiles = g.slab_tiles();
    const VoxLayout L = vox_layout(n, C, ntiles, nisect);
    float4 *rec = reinterpret_cast<float4 *>(static_cast<char *>(ws) + L.rec);
    cudaError_t err;
    if ((err = cudaMemsetAsync(pos_grad, 0, sizeof(float) * 4 * (size_t)n, stream))) return err;
    if ((err = cudaMemsetAsync(conic_grad, 0, sizeof(float) * 6 * (size_t)n, stream))) return err;
    if ((err = cudaMemsetAsync(int_grad, 0, sizeof(float) * C * (size_t)n, stream))) return err;
    if (n <= 0 || ntiles == 0 || nisect <= 0) return cudaSuccess;
    if ((err = launch_prep(n, C, pos_radii, conics, intens, rec, stream))) return err;
    const int2 *bins = reinterpret_cast<const int2 *>(tile_bins);
    const float2 *cq = reinterpret_cast<const float2 *>(conics);
    const unsigned grid = (unsigned)ntiles;
#define GSV_BWDV(Cc)                                                         \
    vox_bwd_voxel_kernel<Cc><<<grid, kVoxThreads, 0, stream>>>(              \
        g, bins, ids, rec, cq, grad, pos_grad, conic_grad, int_grad)
    profile_mark(kProfBackwardVoxel, false, stream);
    switch (C) {
        case 1: GSV_BWDV(1); break;
        case 2: GSV_BWDV(2); break;
        case 3: GSV_BWDV(3); break;
        case 4: GSV_BWDV(4); break;
        default: return cudaErrorInvalidValue;
    }
    profile_mark(kProfBackwardVoxel, true, stream);
#undef GSV_BWDV
    count_launches(1);
    return cudaGetLastError();
}

}  // namespace gsv
