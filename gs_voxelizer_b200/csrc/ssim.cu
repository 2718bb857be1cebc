// 3D SSIM and 3D total-variation losses for volumes in planar layout
// [channels][D][H][W] (W fastest), the losses FaCT-GS-style training puts
// around the voxelizer (the reference's own tests drive it through a 3D SSIM,
// test/test_gs_voxelizer.py:62, test/compare_speed.py:174).
//
// SSIM (Wang, Bovik, Sheikh, Simoncelli 2004, "Image quality assessment:
// from error visibility to structural similarity"), in 3D: local statistics
// under an 11^3 separable Gaussian window (sigma 1.5, normalised), zero
// padding outside the volume, constants C1 = 0.01^2 and C2 = 0.03^2;
//   S = (2 mu_x mu_y + C1)(2 s_xy + C2) / ((mu_x^2 + mu_y^2 + C1)(s_x^2 + s_y^2 + C2)),
// and the loss value is the mean of S over all voxels and channels. With
// the window w, mu_x = w * x, E_xx = w * x^2, E_xy = w * (x y), so
//   dL/dx(p) = (w * G_mu)(p) + 2 x(p) (w * G_xx)(p) + y(p) (w * G_xy)(p)
// where G_mu, G_xx, G_xy are dL/dS times the partial derivatives of S with
// respect to mu_x, E_xx and E_xy at each voxel (the window is symmetric, so
// its adjoint is itself). The forward writes the three G maps for
// dL/dS = 1/N; the backward blurs them and scales by the incoming gradient.
//
// Both kernels stream along z: a CTA owns a 16 x 16 (y, x) output tile and
// a run of 32 z-planes; per input plane it loads the tile with a 5-voxel
// halo into shared memory, blurs along x, then y, and keeps the last 11
// 2D-blurred planes of every map in a per-thread ring in registers, from
// which the z-blur of the output plane 5 behind is formed. Every input
// voxel is read from global memory (1 + 10/16)^2 (1 + 10/32) times, mostly
// from L2; shared-memory traffic and the 3 x 11 taps per map set the cost.
//
// TV (Rudin, Osher, Fatemi 1992), isotropic with a smoothing epsilon, or
// anisotropic: forward differences d_a(v) = x(v + e_a) - x(v) inside the
// volume (0 across the far boundary);
//   iso:   TV = mean_v sqrt(dx^2 + dy^2 + dz^2 + eps)
//   aniso: TV = mean_v (|dx| + |dy| + |dz|)
// One kernel writes the value's per-block partial sums and the gradient.
#include <cmath>

#include "common.cuh"

namespace gsv {

namespace {

constexpr int kSsR = 5;              // window radius (11 taps)
constexpr int kSsTaps = 2 * kSsR + 1;
constexpr int kSsT = 16;             // output tile edge (y and x)
constexpr int kSsIn = kSsT + 2 * kSsR;  // 26: input tile edge with halo
constexpr int kSsZ = 32;             // output z-planes per CTA
constexpr int kSsThreads = kSsT * kSsT;

struct SsWindow {
    float w[kSsTaps];
};

// Partial sums (one per CTA) -> out[0] = sum * scale, in a fixed order.
__global__ void __launch_bounds__(1024)
ss_finish_kernel(int n, const float *__restrict__ part, double scale,
                 float *__restrict__ out) {
    __shared__ double red[32];
    double s = 0.0;
    for (int i = threadIdx.x; i < n; i += blockDim.x) s += (double)part[i];
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
    __syncthreads();
    if (threadIdx.x < 32) {
        s = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.0;
        for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
        if (threadIdx.x == 0) out[0] = (float)(s * scale);
    }
}

__device__ __forceinline__ float block_sum(float v, float *red) {
    const int t = threadIdx.y * blockDim.x + threadIdx.x;
    const int nw = (int)(blockDim.x * blockDim.y) >> 5;
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if ((t & 31) == 0) red[t >> 5] = v;
    __syncthreads();
    float s = 0.f;
    if (t == 0)
        for (int k = 0; k < nw; ++k) s += red[k];
    return s;  // valid in thread (0, 0)
}

// product maps [NM][26][27], rounded up so that what follows is 16-B aligned
__host__ __device__ constexpr int pm_floats(int nm) {
    return (nm * kSsIn * (kSsIn + 1) + 3) & ~3;
}

// NM maps blurred by the window, streamed along z. For each input plane the
// caller's load(inside, zi, yi, xi, vals[NIN]) gives the NIN source values
// of a voxel (zero outside the volume); prod(vals, m) forms map m from them.
// emit(z, y, x, blurred[NM]) is called for every output voxel of the CTA's
// run inside the volume. The last 11 y-blurred planes of the thread's
// column are kept in registers; the plane loop is unrolled by 11 so that
// every ring slot is a compile-time index.
template <int NIN, int NM, class Load, class Prod, class Emit>
__device__ __forceinline__ void blur_stream(int D, int H, int W, int y0,
                                            int x0, int z0, int z1,
                                            const SsWindow &win, float *smem,
                                            Load load, Prod prod, Emit emit) {
    constexpr int kRow = kSsIn + 1;                          // padded row
    float *pm = smem;                                        // [NM][26][27]
    float *xb = pm + pm_floats(NM);                          // [NM][26][16]
    const int tid = threadIdx.x, ty = tid / kSsT, tx = tid % kSsT;
    float ring[kSsTaps][NM];
    const int zend = z1 + kSsR;
    // the thread's (up to 3) positions of the 26 x 26 input plane; the next
    // plane's values are loaded while this plane is blurred
    constexpr int kPer = (kSsIn * kSsIn + kSsThreads - 1) / kSsThreads;
    float nv[kPer][NIN];
    auto fetch = [&](int zi) {
#pragma unroll
        for (int q = 0; q < kPer; ++q) {
            const int e = tid + q * kSsThreads;
            const int r = e / kSsIn, c = e % kSsIn;
            const int yi = y0 - kSsR + r, xi = x0 - kSsR + c;
            const bool inside = e < kSsIn * kSsIn && zi >= 0 && zi < D &&
                                yi >= 0 && yi < H && xi >= 0 && xi < W;
            load(inside, zi, yi, xi, nv[q]);
        }
    };
    fetch(z0 - kSsR);
    for (int zb = z0 - kSsR; zb < zend; zb += kSsTaps) {
#pragma unroll
        for (int j = 0; j < kSsTaps; ++j) {
            const int zi = zb + j;
            if (zi >= zend) break;  // uniform over the CTA
            // 1. input plane with halo, as the NM product maps
#pragma unroll
            for (int q = 0; q < kPer; ++q) {
                const int e = tid + q * kSsThreads;
                if (e < kSsIn * kSsIn) {
                    const int r = e / kSsIn, c = e % kSsIn;
#pragma unroll
                    for (int m = 0; m < NM; ++m)
                        pm[(m * kSsIn + r) * kRow + c] = prod(nv[q], m);
                }
            }
            if (zi + 1 < zend) fetch(zi + 1);
            __syncthreads();
            // 2. blur along x: tasks of 4 consecutive outputs of one row of
            //    one map, from a 14-value register window
            for (int e = tid; e < NM * kSsIn * (kSsT / 4); e += kSsThreads) {
                const int m = e / (kSsIn * (kSsT / 4)), rest = e % (kSsIn * (kSsT / 4));
                const int r = rest / (kSsT / 4), c0 = 4 * (rest % (kSsT / 4));
                const float *src = pm + (m * kSsIn + r) * kRow + c0;
                float v[4 + 2 * kSsR];
#pragma unroll
                for (int k = 0; k < 4 + 2 * kSsR; ++k) v[k] = src[k];
                float acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
                for (int k = 0; k < kSsTaps; ++k)
#pragma unroll
                    for (int q = 0; q < 4; ++q) acc[q] = fmaf(win.w[k], v[q + k], acc[q]);
                *reinterpret_cast<float4 *>(xb + (m * kSsIn + r) * kSsT + c0) =
                    make_float4(acc[0], acc[1], acc[2], acc[3]);
            }
            __syncthreads();
            // 3. blur along y for this thread's column, into ring slot j
#pragma unroll
            for (int m = 0; m < NM; ++m) {
                float acc = 0.f;
#pragma unroll
                for (int k = 0; k < kSsTaps; ++k)
                    acc = fmaf(win.w[k], xb[(m * kSsIn + ty + k) * kSsT + tx], acc);
                ring[j][m] = acc;
            }
            // 4. blur along z: output plane zo = zi - 5 from planes zi - 10 ..
            //    zi, held in slots (j + 1) % 11 .. j
            const int zo = zi - kSsR;
            if (zo >= z0) {
                float acc[NM];
#pragma unroll
                for (int m = 0; m < NM; ++m) acc[m] = 0.f;
#pragma unroll
                for (int k = 0; k < kSsTaps; ++k)
#pragma unroll
                    for (int m = 0; m < NM; ++m)
                        acc[m] = fmaf(win.w[k], ring[(j + 1 + k) % kSsTaps][m], acc[m]);
                const int y = y0 + ty, x = x0 + tx;
                if (zo < D && y < H && x < W) emit(zo, y, x, acc);
            }
            __syncthreads();  // the product maps and xb are rewritten next
        }
    }
}

constexpr int ss_smem_floats(int nm) {
    return pm_floats(nm) + nm * kSsIn * kSsT;
}

// Forward: mean SSIM partials per CTA and the three G maps (dL/dS = 1/N).
__global__ void __launch_bounds__(kSsThreads)
ssim_fwd_kernel(int D, int H, int W, int zchunks, const float *__restrict__ img1,
                const float *__restrict__ img2, float C1, float C2, float inv_n,
                SsWindow win, float *__restrict__ gmu, float *__restrict__ gxx,
                float *__restrict__ gxy, float *__restrict__ part) {
    extern __shared__ float ss_smem[];
    __shared__ float red[kSsThreads / 32];
    const int ch = blockIdx.z / zchunks, zc = blockIdx.z % zchunks;
    const size_t plane = (size_t)H * W, vol = plane * D;
    const float *a = img1 + ch * vol, *b = img2 + ch * vol;
    const size_t off = ch * vol;
    const int y0 = blockIdx.y * kSsT, x0 = blockIdx.x * kSsT;
    const int z0 = zc * kSsZ, z1 = min(D, z0 + kSsZ);
    float lsum = 0.f;
    blur_stream<2, 5>(
        D, H, W, y0, x0, z0, z1, win, ss_smem,
        [&](bool inside, int z, int y, int x, float (&v)[2]) {
            const size_t i = (size_t)z * plane + (size_t)y * W + x;
            v[0] = inside ? __ldg(a + i) : 0.f;
            v[1] = inside ? __ldg(b + i) : 0.f;
        },
        [](const float (&v)[2], int m) {
            return m == 0 ? v[0] : m == 1 ? v[1] : m == 2 ? v[0] * v[0]
                 : m == 3 ? v[1] * v[1] : v[0] * v[1];
        },
        [&](int z, int y, int x, const float (&s)[5]) {
            const float mx = s[0], my = s[1];
            const float sxx = s[2] - mx * mx, syy = s[3] - my * my,
                        sxy = s[4] - mx * my;
            const float A1 = 2.f * mx * my + C1, A2 = 2.f * sxy + C2;
            const float B1 = mx * mx + my * my + C1, B2 = sxx + syy + C2;
            const float inv = 1.f / (B1 * B2);
            const float S = A1 * A2 * inv;
            lsum += S;
            const size_t i = off + (size_t)z * plane + (size_t)y * W + x;
            gmu[i] = inv_n * (2.f * my * (A2 - A1) * inv +
                              2.f * mx * S * (1.f / B2 - 1.f / B1));
            gxx[i] = inv_n * (-S / B2);
            gxy[i] = inv_n * (2.f * A1 * inv);
        });
    const float s = block_sum(lsum, red);
    const unsigned cta = (blockIdx.z * gridDim.y + blockIdx.y) * gridDim.x + blockIdx.x;
    if (threadIdx.x == 0) part[cta] = s;
}

// Backward: dL/dx = g * (w*G_mu + 2 x w*G_xx + y w*G_xy).
__global__ void __launch_bounds__(kSsThreads)
ssim_bwd_kernel(int D, int H, int W, int zchunks, const float *__restrict__ img1,
                const float *__restrict__ img2, SsWindow win,
                const float *__restrict__ gmu, const float *__restrict__ gxx,
                const float *__restrict__ gxy, const float *__restrict__ grad_out,
                float *__restrict__ grad) {
    extern __shared__ float ss_smem[];
    const int ch = blockIdx.z / zchunks, zc = blockIdx.z % zchunks;
    const size_t plane = (size_t)H * W, vol = plane * D;
    const size_t off = ch * vol;
    const int y0 = blockIdx.y * kSsT, x0 = blockIdx.x * kSsT;
    const int z0 = zc * kSsZ, z1 = min(D, z0 + kSsZ);
    const float g = __ldg(grad_out);
    blur_stream<3, 3>(
        D, H, W, y0, x0, z0, z1, win, ss_smem,
        [&](bool inside, int z, int y, int x, float (&v)[3]) {
            const size_t i = off + (size_t)z * plane + (size_t)y * W + x;
            v[0] = inside ? __ldg(gmu + i) : 0.f;
            v[1] = inside ? __ldg(gxx + i) : 0.f;
            v[2] = inside ? __ldg(gxy + i) : 0.f;
        },
        [](const float (&v)[3], int m) { return v[m]; },
        [&](int z, int y, int x, const float (&s)[3]) {
            const size_t i = off + (size_t)z * plane + (size_t)y * W + x;
            const float xa = __ldg(img1 + i), yb = __ldg(img2 + i);
            grad[i] = g * (s[0] + 2.f * xa * s[1] + yb * s[2]);
        });
}

// TV: value partials per block and the gradient (grad_out scaled). Block
// (32, 8) over (x, y); each thread marches down a run of kTvZ z-planes of
// its column, so the differences at v - e_z are the previous plane's and
// every value of the next plane it needs is loaded once: per voxel 3 loads
// for the value, 7 with the gradient. Grid z = runs * channels.
constexpr int kTvZ = 8;

template <bool ISO>
__device__ __forceinline__ float tv_term(float dx, float dy, float dz, float eps) {
    return ISO ? sqrtf(dx * dx + dy * dy + dz * dz + eps)
               : fabsf(dx) + fabsf(dy) + fabsf(dz);
}

__device__ __forceinline__ float sgnf(float v) { return (float)((v > 0.f) - (v < 0.f)); }

template <bool ISO>
__global__ void __launch_bounds__(256)
tv_kernel(int D, int H, int W, int runs, const float *__restrict__ x, float eps,
          float inv_n, const float *__restrict__ grad_out,
          float *__restrict__ grad, float *__restrict__ part) {
    __shared__ float red[8];
    const int xx = blockIdx.x * 32 + threadIdx.x, y = blockIdx.y * 8 + threadIdx.y;
    const int run = blockIdx.z % runs, ch = blockIdx.z / runs;
    const int z0 = run * kTvZ, z1 = min(D, z0 + kTvZ);
    const size_t plane = (size_t)H * W;
    float lsum = 0.f;
    if (xx < W && y < H) {
        const float *xc = x + (size_t)ch * plane * D;
        const size_t col = (size_t)y * W + xx;
        const bool hx = xx + 1 < W, hy = y + 1 < H, bx = xx > 0, by = y > 0;
        const float g = grad ? __ldg(grad_out) * inv_n : 0.f;
        // value at (z, column + off), 0 outside [0, D)
        auto at = [&](int z, long long off) {
            return (z >= 0 && z < D) ? __ldg(xc + (size_t)z * plane + col + off) : 0.f;
        };
        float c = at(z0, 0);                     // x(v)
        float a = bx ? at(z0, -1) : 0.f;         // x(v - ex)
        float b = by ? at(z0, -W) : 0.f;         // x(v - ey)
        // the voxel behind in z: its differences dz and its term
        float pdz = 0.f, pt = 1.f;
        if (grad && z0 > 0) {
            const float pc = at(z0 - 1, 0);
            const float pdx = hx ? at(z0 - 1, 1) - pc : 0.f;
            const float pdy = hy ? at(z0 - 1, W) - pc : 0.f;
            pdz = c - pc;
            pt = tv_term<ISO>(pdx, pdy, pdz, eps);
        }
        for (int z = z0; z < z1; ++z) {
            const bool hz = z + 1 < D;
            const float cz = hz ? at(z + 1, 0) : 0.f;  // next plane's c
            const float dx = hx ? at(z, 1) - c : 0.f;
            const float dy = hy ? at(z, W) - c : 0.f;
            const float dz = hz ? cz - c : 0.f;
            const float t = tv_term<ISO>(dx, dy, dz, eps);
            lsum += t;
            float az = 0.f, bz = 0.f;
            if (grad) {
                float gr = ISO ? -(dx + dy + dz) / t : -(sgnf(dx) + sgnf(dy) + sgnf(dz));
                if (bx) {  // term of v - ex: dx(v - ex) = x(v) - x(v - ex)
                    az = hz ? at(z + 1, -1) : 0.f;
                    const float ex = c - a;
                    const float ey = hy ? at(z, W - 1) - a : 0.f;
                    const float ez = hz ? az - a : 0.f;
                    gr += ISO ? ex / tv_term<true>(ex, ey, ez, eps) : sgnf(ex);
                }
                if (by) {  // term of v - ey
                    bz = hz ? at(z + 1, -W) : 0.f;
                    const float fx = hx ? at(z, 1 - W) - b : 0.f;
                    const float fy = c - b;
                    const float fz = hz ? bz - b : 0.f;
                    gr += ISO ? fy / tv_term<true>(fx, fy, fz, eps) : sgnf(fy);
                }
                if (z > 0)  // term of v - ez (the previous plane's)
                    gr += ISO ? pdz / pt : sgnf(pdz);
                grad[(size_t)ch * plane * D + (size_t)z * plane + col] = g * gr;
                pdz = dz;
                pt = t;
            } else {
                if (bx && hz) az = at(z + 1, -1);
                if (by && hz) bz = at(z + 1, -W);
            }
            c = cz;
            a = az;
            b = bz;
        }
    }
    if (part) {
        const float s = block_sum(lsum, red);
        const unsigned blk = (blockIdx.z * gridDim.y + blockIdx.y) * gridDim.x + blockIdx.x;
        if (threadIdx.x == 0 && threadIdx.y == 0) part[blk] = s;
    }
}

}  // namespace

SsWindowHost ssim_window(double sigma) {
    SsWindowHost w;
    double tot = 0.0, v[kSsTaps];
    for (int k = 0; k < kSsTaps; ++k) {
        const double d = k - kSsR;
        v[k] = std::exp(-d * d / (2.0 * sigma * sigma));
        tot += v[k];
    }
    for (int k = 0; k < kSsTaps; ++k) w.w[k] = (float)(v[k] / tot);
    return w;
}

static dim3 ssim_grid(int nch, int D, int H, int W, int &zchunks) {
    zchunks = (D + kSsZ - 1) / kSsZ;
    return dim3((unsigned)((W + kSsT - 1) / kSsT), (unsigned)((H + kSsT - 1) / kSsT),
                (unsigned)(zchunks * nch));
}

size_t ssim_workspace_bytes(int nch, int D, int H, int W) {
    int zc;
    const dim3 g = ssim_grid(nch, D, H, W, zc);
    const size_t nvox = (size_t)nch * D * H * W;
    return ((3 * nvox * sizeof(float) + 255) & ~size_t(255)) +
           (((size_t)g.x * g.y * g.z * sizeof(float) + 255) & ~size_t(255));
}

cudaError_t launch_ssim_forward(int nch, int D, int H, int W, const float *img1,
                                const float *img2, float C1, float C2,
                                const SsWindowHost &w, float *ssim_out, void *ws,
                                cudaStream_t stream) {
    int zc;
    const dim3 grid = ssim_grid(nch, D, H, W, zc);
    const size_t nvox = (size_t)nch * D * H * W;
    float *gmu = static_cast<float *>(ws), *gxx = gmu + nvox, *gxy = gxx + nvox;
    float *part = reinterpret_cast<float *>(static_cast<char *>(ws) +
                                            ((3 * nvox * sizeof(float) + 255) & ~size_t(255)));
    SsWindow win;
    for (int k = 0; k < kSsTaps; ++k) win.w[k] = w.w[k];
    constexpr int smem = ss_smem_floats(5) * (int)sizeof(float);
    static bool attr = false;
    if (!attr) {
        cudaError_t e = cudaFuncSetAttribute(
            ssim_fwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        if (e) return e;
        attr = true;
    }
    ssim_fwd_kernel<<<grid, kSsThreads, smem, stream>>>(
        D, H, W, zc, img1, img2, C1, C2, (float)(1.0 / (double)nvox), win, gmu,
        gxx, gxy, part);
    const int nparts = (int)(grid.x * grid.y * grid.z);
    ss_finish_kernel<<<1, 1024, 0, stream>>>(nparts, part, 1.0 / (double)nvox,
                                             ssim_out);
    count_launches(2);
    return cudaGetLastError();
}

cudaError_t launch_ssim_backward(int nch, int D, int H, int W, const float *img1,
                                 const float *img2, const SsWindowHost &w,
                                 const float *grad_out, const void *ws,
                                 float *grad, cudaStream_t stream) {
    int zc;
    const dim3 grid = ssim_grid(nch, D, H, W, zc);
    const size_t nvox = (size_t)nch * D * H * W;
    const float *gmu = static_cast<const float *>(ws), *gxx = gmu + nvox,
                *gxy = gxx + nvox;
    SsWindow win;
    for (int k = 0; k < kSsTaps; ++k) win.w[k] = w.w[k];
    constexpr int smem = ss_smem_floats(3) * (int)sizeof(float);
    static bool attr = false;
    if (!attr) {
        cudaError_t e = cudaFuncSetAttribute(
            ssim_bwd_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        if (e) return e;
        attr = true;
    }
    ssim_bwd_kernel<<<grid, kSsThreads, smem, stream>>>(
        D, H, W, zc, img1, img2, win, gmu, gxx, gxy, grad_out, grad);
    count_launches(1);
    return cudaGetLastError();
}

static dim3 tv_grid(int nch, int D, int H, int W) {
    return dim3((unsigned)((W + 31) / 32), (unsigned)((H + 7) / 8),
                (unsigned)(((D + kTvZ - 1) / kTvZ) * nch));
}

size_t tv_workspace_bytes(int nch, int D, int H, int W) {
    const dim3 g = tv_grid(nch, D, H, W);
    return ((size_t)g.x * g.y * g.z * sizeof(float) + 255) & ~size_t(255);
}

cudaError_t launch_tv(int nch, int D, int H, int W, const float *x, int iso,
                      float eps, float *value_out, const float *grad_out,
                      float *grad, void *ws, cudaStream_t stream) {
    const size_t total = (size_t)nch * D * H * W;
    const dim3 grid = tv_grid(nch, D, H, W);
    float *part = value_out ? static_cast<float *>(ws) : nullptr;
    const float inv_n = (float)(1.0 / (double)total);
    if (iso)
        tv_kernel<true><<<grid, dim3(32, 8), 0, stream>>>(D, H, W, (D + kTvZ - 1) / kTvZ, x, eps, inv_n,
                                                          grad_out, grad, part);
    else
        tv_kernel<false><<<grid, dim3(32, 8), 0, stream>>>(D, H, W, (D + kTvZ - 1) / kTvZ, x, eps, inv_n,
                                                           grad_out, grad, part);
    count_launches(1);
    if (value_out) {
        ss_finish_kernel<<<1, 1024, 0, stream>>>((int)(grid.x * grid.y * grid.z),
                                                 part, 1.0 / (double)total, value_out);
        count_launches(1);
    }
    return cudaGetLastError();
}

}  // namespace gsv
