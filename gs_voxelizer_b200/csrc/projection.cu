// Projection: optimisation parameters -> render parameters, and its backward.
//
// Follows gs_voxelizer/cuda/optim_to_render.cu:26-172 (forward) and :186-336
// (backward) plus optim_to_render_helpers.cuh:15-75 of the reference. The
// floating-point expression trees (the order of every product and sum, the
// column-major 3x3 products, the approximate division / sqrt / log that
// --use_fast_math selects) are kept the same as the reference's on purpose:
// tile_min / tile_max / num_tiles_hit are integers truncated from these
// floats, and they must match the reference bit for bit. This file is
// compiled with -use_fast_math for the same reason.
//
// Layout: one thread per Gaussian, 128-thread CTAs. Inputs are read as
// scalars from the packed [N,3] arrays (pos3d, scale3d are 12-byte rows and
// cannot be loaded as float4); outputs are stored as float4 / float2 / int.
#include "common.cuh"

namespace gsv {
namespace {

// Column-major 3x3 matrix: m[c][r] is column c, row r (the GLM convention of
// the reference).
struct Mat3 {
    float m[3][3];
};

__device__ __forceinline__ Mat3 mul(const Mat3 &a, const Mat3 &b) {
    Mat3 o;
#pragma unroll
    for (int c = 0; c < 3; ++c)
#pragma unroll
        for (int r = 0; r < 3; ++r)
            o.m[c][r] = a.m[0][r] * b.m[c][0] + a.m[1][r] * b.m[c][1] +
                        a.m[2][r] * b.m[c][2];
    return o;
}

__device__ __forceinline__ Mat3 transpose(const Mat3 &a) {
    Mat3 o;
#pragma unroll
    for (int c = 0; c < 3; ++c)
#pragma unroll
        for (int r = 0; r < 3; ++r) o.m[c][r] = a.m[r][c];
    return o;
}

// diag(d) * a  (left-multiplication by a diagonal matrix scales rows)
__device__ __forceinline__ Mat3 diag_mul(const float d[3], const Mat3 &a) {
    Mat3 o;
#pragma unroll
    for (int c = 0; c < 3; ++c)
#pragma unroll
        for (int r = 0; r < 3; ++r) o.m[c][r] = d[r] * a.m[c][r];
    return o;
}

// a * diag(d)  (right-multiplication by a diagonal matrix scales columns)
__device__ __forceinline__ Mat3 mul_diag(const Mat3 &a, const float d[3]) {
    Mat3 o;
#pragma unroll
    for (int c = 0; c < 3; ++c)
#pragma unroll
        for (int r = 0; r < 3; ++r) o.m[c][r] = a.m[c][r] * d[c];
    return o;
}

// Rotation matrix of the quaternion stored (w, x, y, z) in a float4's
// (.x, .y, .z, .w), normalised with rsqrt (helpers.cuh:15-37).
struct Quat {
    float w, x, y, z;
};

__device__ __forceinline__ Quat normalise(float4 q) {
    const float inv = rsqrtf(q.w * q.w + q.x * q.x + q.y * q.y + q.z * q.z);
    Quat n;
    n.w = q.x * inv;
    n.x = q.y * inv;
    n.y = q.z * inv;
    n.z = q.w * inv;
    return n;
}

__device__ __forceinline__ Mat3 rotation(const Quat &q) {
    const float w = q.w, x = q.x, y = q.y, z = q.z;
    Mat3 R;
    R.m[0][0] = 1.f - 2.f * (y * y + z * z);
    R.m[0][1] = 2.f * (x * y - w * z);
    R.m[0][2] = 2.f * (x * z + w * y);
    R.m[1][0] = 2.f * (x * y + w * z);
    R.m[1][1] = 1.f - 2.f * (x * x + z * z);
    R.m[1][2] = 2.f * (y * z - w * x);
    R.m[2][0] = 2.f * (x * z - w * y);
    R.m[2][1] = 2.f * (y * z + w * x);
    R.m[2][2] = 1.f - 2.f * (x * x + y * y);
    return R;
}

// Voxel-space covariance (S R)^T (S R) scaled by diag(1/voxel size).
// inv_vox = (1/vx, 1/vy, 1/vz) in matrix-axis order (axis 0 = x).
__device__ __forceinline__ Mat3 voxel_covariance(const float s[3],
                                                 const Mat3 &R,
                                                 const float inv_vox[3]) {
    const Mat3 M = diag_mul(s, R);
    const Mat3 cov = mul(transpose(M), M);
    return mul_diag(diag_mul(inv_vox, cov), inv_vox);
}

__device__ __forceinline__ int tile_floor(float v, int bound) {
    return min(bound, max(0, (int)(v / (float)kTile)));
}

template <int C>
__global__ void __launch_bounds__(128)
project_fwd_kernel(int n, const float *__restrict__ pos3d,
                   const float *__restrict__ scale3d,
                   const float4 *__restrict__ quat,
                   const float *__restrict__ intensities, int vz, int vy,
                   int vx, int tiles_x, int tiles_y, int tiles_z, float wz,
                   float wy, float wx, float cz, float cy, float cx,
                   float4 *__restrict__ pos_radii_out,
                   float2 *__restrict__ conics_out,
                   int *__restrict__ tile_min_out,
                   int *__restrict__ tile_max_out,
                   int *__restrict__ num_tiles_out) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;

    // voxel edge lengths per axis (z, y, x as in the reference's float3)
    const float vox_z = wz / (float)vz;
    const float vox_y = wy / (float)vy;
    const float vox_x = wx / (float)vx;

    const float p0 = pos3d[3 * i + 0], p1 = pos3d[3 * i + 1],
                p2 = pos3d[3 * i + 2];
    const float px = (p0 - cx + (wx * 0.5f)) / vox_x;
    const float py = (p1 - cy + (wy * 0.5f)) / vox_y;
    const float pz = (p2 - cz + (wz * 0.5f)) / vox_z;

    const float s[3] = {scale3d[3 * i + 0], scale3d[3 * i + 1],
                        scale3d[3 * i + 2]};
    const Mat3 R = rotation(normalise(quat[i]));
    const float inv_vox[3] = {1.f / vox_x, 1.f / vox_y, 1.f / vox_z};
    const Mat3 cov = voxel_covariance(s, R, inv_vox);

    const float a = cov.m[0][0], b = cov.m[0][1], c = cov.m[0][2];
    const float d = cov.m[1][1], e = cov.m[1][2], f = cov.m[2][2];
    const float det = a * d * f + 2 * b * c * e - a * e * e - f * b * b -
                      d * c * c;

    float4 pos_out = make_float4(0.f, 0.f, 0.f, 0.f);
    float2 q01 = make_float2(0.f, 0.f), q23 = q01, q45 = q01;
    int3 tmin = make_int3(0, 0, 0), tmax = tmin;
    int hit = 0;

    if (det != 0.0f) {
        const float inv_det = 1.0f / det;
        const float qa = inv_det * (d * f - e * e);
        const float qb = inv_det * (c * e - b * f);
        const float qc = inv_det * (b * e - c * d);
        const float qd = inv_det * (a * f - c * c);
        const float qe = inv_det * (b * c - a * e);
        const float qf = inv_det * (a * d - b * b);

        // cull radius from the largest scale, in voxels
        const float radius =
            ceil((3.f * max(s[0], max(s[1], s[2]))) /
                 min(vox_x, min(vox_y, vox_z)));

        float mean = 0.f;
#pragma unroll
        for (int k = 0; k < C; ++k) mean += intensities[i * C + k];
        mean /= C;
        // extent where alpha * mean reaches 1e-6, capped at 3 sigma
        const float log_thr = logf(mean * (1 / 0.000001f));
        const float extent = min(3.f, sqrtf(2.0f * log_thr));
        const float rx = max(0.0f, (sqrtf(a) * extent) - 0.5f);
        const float ry = max(0.0f, (sqrtf(d) * extent) - 0.5f);
        const float rz = max(0.0f, (sqrtf(f) * extent) - 0.5f);

        const bool outside = radius <= 0.f || px + radius < 0.f ||
                             px - radius > (float)(unsigned)vx ||
                             py + radius < 0.f ||
                             py - radius > (float)(unsigned)vy ||
                             pz + radius < 0.f ||
                             pz - radius > (float)(unsigned)vz;
        if (!outside) {
            int3 lo, hi;
            lo.x = tile_floor(px - rx, tiles_x);
            lo.y = tile_floor(py - ry, tiles_y);
            lo.z = tile_floor(pz - rz, tiles_z);
            hi.x = tile_floor(px + rx + (float)(kTile - 1), tiles_x);
            hi.y = tile_floor(py + ry + (float)(kTile - 1), tiles_y);
            hi.z = tile_floor(pz + rz + (float)(kTile - 1), tiles_z);
            const int vol = (hi.x - lo.x) * (hi.y - lo.y) * (hi.z - lo.z);
            if (vol > 0) {
                pos_out = make_float4(px, py, pz, radius);
                q01 = make_float2(qa, qb);
                q23 = make_float2(qc, qd);
                q45 = make_float2(qe, qf);
                tmin = lo;
                tmax = hi;
                hit = vol;
            }
        }
    }
    pos_radii_out[i] = pos_out;
    conics_out[3 * i + 0] = q01;
    conics_out[3 * i + 1] = q23;
    conics_out[3 * i + 2] = q45;
    tile_min_out[3 * i + 0] = tmin.x;
    tile_min_out[3 * i + 1] = tmin.y;
    tile_min_out[3 * i + 2] = tmin.z;
    tile_max_out[3 * i + 0] = tmax.x;
    tile_max_out[3 * i + 1] = tmax.y;
    tile_max_out[3 * i + 2] = tmax.z;
    num_tiles_out[i] = hit;
}

// d(conic)/d(covariance) chain, then back to world space and symmetrised
// (optim_to_render.cu:186-239). The 1e-7 in the denominator regularises
// near-singular covariances exactly as the reference does.
__device__ __forceinline__ Mat3 covariance_grad(const Mat3 &cov,
                                                const float inv_vox[3],
                                                float2 g01, float2 g23,
                                                float2 g45) {
    const float a = cov.m[0][0], b = cov.m[0][1], c = cov.m[0][2];
    const float d = cov.m[1][1], e = cov.m[1][2], f = cov.m[2][2];
    const float det = a * d * f + 2 * b * c * e - a * e * e - f * b * b -
                      d * c * c;
    const float k = 1.0f / ((det * det) + 0.0000001f);
    Mat3 out;
#pragma unroll
    for (int cc = 0; cc < 3; ++cc)
#pragma unroll
        for (int r = 0; r < 3; ++r) out.m[cc][r] = 0.f;
    if (k == 0) return out;

    // partial derivatives of det with respect to a..f
    const float det_a = d * f - e * e;
    const float det_b = 2 * c * e - 2 * f * b;
    const float det_c = 2 * b * e - 2 * d * c;
    const float det_d = a * f - c * c;
    const float det_e = 2 * b * c - 2 * a * e;
    const float det_f = a * d - b * b;
    // cofactors that form the numerators of conic b, c, e
    const float num_b = c * e - b * f;
    const float num_c = b * e - c * d;
    const float num_e = b * c - a * e;

    const float ga = k * (-det_a * det_a * g01.x - num_b * det_a * g01.y -
                          num_c * det_a * g23.x +
                          (f * det - det_d * det_a) * g23.y +
                          (-e * det - num_e * det_a) * g45.x +
                          (d * det - det_f * det_a) * g45.y);
    const float gb = k * (-det_a * det_b * g01.x +
                          (-f * det - num_b * det_b) * g01.y +
                          (e * det - num_c * det_b) * g23.x -
                          det_d * det_b * g23.y +
                          (c * det - num_e * det_b) * g45.x +
                          (-2 * b * det - det_f * det_b) * g45.y);
    const float gc = k * (-det_a * det_c * g01.x +
                          (e * det - num_b * det_c) * g01.y +
                          (-d * det - num_c * det_c) * g23.x +
                          (-2 * c * det - det_d * det_c) * g23.y +
                          (b * det - num_e * det_c) * g45.x -
                          det_f * det_c * g45.y);
    const float gd = k * ((f * det - det_a * det_d) * g01.x -
                          num_b * det_d * g01.y +
                          (-c * det - num_c * det_d) * g23.x -
                          det_d * det_d * g23.y - num_e * det_d * g45.x +
                          (a * det - det_f * det_d) * g45.y);
    const float ge = k * ((-2 * e * det - det_a * det_e) * g01.x +
                          (c * det - num_b * det_e) * g01.y +
                          (b * det - num_c * det_e) * g23.x -
                          det_d * det_e * g23.y +
                          (-a * det - num_e * det_e) * g45.x +
                          -det_f * det_e * g45.y);
    const float gf = k * ((d * det - det_a * det_f) * g01.x +
                          (-b * det - num_b * det_f) * g01.y -
                          num_c * det_f * g23.x +
                          (a * det - det_d * det_f) * g23.y -
                          num_e * det_f * g45.x - det_f * det_f * g45.y);

    Mat3 G;
    G.m[0][0] = ga; G.m[0][1] = gb; G.m[0][2] = gc;
    G.m[1][0] = gb; G.m[1][1] = gd; G.m[1][2] = ge;
    G.m[2][0] = gc; G.m[2][1] = ge; G.m[2][2] = gf;
    // M2 * G * M2^T with M2 = diag(inv_vox)
    const Mat3 W = mul_diag(diag_mul(inv_vox, G), inv_vox);
    const Mat3 Wt = transpose(W);
#pragma unroll
    for (int cc = 0; cc < 3; ++cc)
#pragma unroll
        for (int r = 0; r < 3; ++r)
            out.m[cc][r] = 0.5f * (W.m[cc][r] + Wt.m[cc][r]);
    return out;
}

__global__ void __launch_bounds__(128)
project_bwd_kernel(int n, const float *__restrict__ pos3d,
                   const float *__restrict__ scale3d,
                   const float4 *__restrict__ quat, int vz, int vy, int vx,
                   float wz, float wy, float wx,
                   const float4 *__restrict__ pos_radii_grad,
                   const float2 *__restrict__ conics_grad,
                   const float4 *__restrict__ pos_radii,
                   float *__restrict__ pos_grad_out,
                   float *__restrict__ scale_grad_out,
                   float4 *__restrict__ quat_grad_out) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    (void)pos3d;

    float gp[3] = {0.f, 0.f, 0.f}, gs[3] = {0.f, 0.f, 0.f};
    float4 gq = make_float4(0.f, 0.f, 0.f, 0.f);

    if (pos_radii[i].w > 0) {
        const float2 g01 = conics_grad[3 * i + 0];
        const float2 g23 = conics_grad[3 * i + 1];
        const float2 g45 = conics_grad[3 * i + 2];

        const float vox_z = wz / (float)(unsigned)vz;
        const float vox_y = wy / (float)(unsigned)vy;
        const float vox_x = wx / (float)(unsigned)vx;

        const float s[3] = {scale3d[3 * i + 0], scale3d[3 * i + 1],
                            scale3d[3 * i + 2]};
        const float4 qraw = quat[i];
        const Quat q = normalise(qraw);
        const Mat3 R = rotation(q);
        const float inv_vox[3] = {1.f / vox_x, 1.f / vox_y, 1.f / vox_z};
        const Mat3 cov = voxel_covariance(s, R, inv_vox);
        const Mat3 cg = covariance_grad(cov, inv_vox, g01, g23, g45);

        // gradient w.r.t. the symmetric covariance, off-diagonals halved
        Mat3 dS;
#pragma unroll
        for (int c = 0; c < 3; ++c)
#pragma unroll
            for (int r = 0; r < 3; ++r)
                dS.m[c][r] = (c == r) ? cg.m[c][r] : 0.5f * cg.m[c][r];

        // dL/dR = 2 S R dS   (S = diag(s))
        float s2[3] = {2.0f * s[0], 2.0f * s[1], 2.0f * s[2]};
        const Mat3 Rg = mul(diag_mul(s2, R), dS);
        Mat3 Rgt = transpose(Rg);
        const Mat3 Rt = transpose(R);
#pragma unroll
        for (int k = 0; k < 3; ++k)
            gs[k] = Rt.m[k][0] * Rgt.m[k][0] + Rt.m[k][1] * Rgt.m[k][1] +
                    Rt.m[k][2] * Rgt.m[k][2];
#pragma unroll
        for (int k = 0; k < 3; ++k)
#pragma unroll
            for (int r = 0; r < 3; ++r) Rgt.m[k][r] *= s[k];

        // The reference multiplies the incoming pixel-space position gradient
        // by the voxel size (optim_to_render.cu:329-331); kept as is.
        const float4 gpr = pos_radii_grad[i];
        gp[0] = gpr.x * vox_x;
        gp[1] = gpr.y * vox_y;
        gp[2] = gpr.z * vox_z;

        // dL/dquat from dL/dR (helpers.cuh:51-75), quaternion (w,x,y,z)
        const float w = q.w, x = q.x, y = q.y, z = q.z;
        const Mat3 &v = Rgt;
        gq.x = 2 * z * (v.m[0][1] - v.m[1][0]) +
               2 * y * (v.m[2][0] - v.m[0][2]) +
               2 * x * (v.m[1][2] - v.m[2][1]);
        gq.y = 2 * y * (v.m[1][0] + v.m[0][1]) +
               2 * z * (v.m[2][0] + v.m[0][2]) +
               2 * w * (v.m[1][2] - v.m[2][1]) -
               4 * x * (v.m[2][2] + v.m[1][1]);
        gq.z = 2 * x * (v.m[1][0] + v.m[0][1]) +
               2 * w * (v.m[2][0] - v.m[0][2]) +
               2 * z * (v.m[1][2] + v.m[2][1]) -
               4 * y * (v.m[2][2] + v.m[0][0]);
        gq.w = 2 * w * (v.m[0][1] - v.m[1][0]) +
               2 * x * (v.m[2][0] + v.m[0][2]) +
               2 * y * (v.m[1][2] + v.m[2][1]) -
               4 * z * (v.m[1][1] + v.m[0][0]);
    }
    pos_grad_out[3 * i + 0] = gp[0];
    pos_grad_out[3 * i + 1] = gp[1];
    pos_grad_out[3 * i + 2] = gp[2];
    scale_grad_out[3 * i + 0] = gs[0];
    scale_grad_out[3 * i + 1] = gs[1];
    scale_grad_out[3 * i + 2] = gs[2];
    quat_grad_out[i] = gq;
}

}  // namespace

cudaError_t launch_project_fwd(int n, int channels, const float *pos3d,
                               const float *scale3d, const float *quat,
                               const float *intensities, const int vol[3],
                               const float world[3], const float center[3],
                               float *pos_radii, float *conics, int *tile_min,
                               int *tile_max, int *num_tiles,
                               cudaStream_t stream) {
    if (n <= 0) return cudaSuccess;
    const int tx = (vol[2] + kTile - 1) / kTile;
    const int ty = (vol[1] + kTile - 1) / kTile;
    const int tz = (vol[0] + kTile - 1) / kTile;
    const dim3 grid((n + 127) / 128), block(128);
#define GSV_PROJ(Cc)                                                        \
    project_fwd_kernel<Cc><<<grid, block, 0, stream>>>(                     \
        n, pos3d, scale3d, reinterpret_cast<const float4 *>(quat),          \
        intensities, vol[0], vol[1], vol[2], tx, ty, tz, world[0],          \
        world[1], world[2], center[0], center[1], center[2],               \
        reinterpret_cast<float4 *>(pos_radii),                              \
        reinterpret_cast<float2 *>(conics), tile_min, tile_max, num_tiles)
    switch (channels) {
        case 1: GSV_PROJ(1); break;
        case 2: GSV_PROJ(2); break;
        case 3: GSV_PROJ(3); break;
        case 4: GSV_PROJ(4); break;
        default: return cudaErrorInvalidValue;
    }
#undef GSV_PROJ
    count_launches(1);
    return cudaGetLastError();
}

cudaError_t launch_project_bwd(int n, const float *pos3d, const float *scale3d,
                               const float *quat, const int vol[3],
                               const float world[3], const float *pos_radii_grad,
                               const float *conics_grad, const float *pos_radii,
                               float *pos_grad, float *scale_grad,
                               float *quat_grad, cudaStream_t stream) {
    if (n <= 0) return cudaSuccess;
    project_bwd_kernel<<<(n + 127) / 128, 128, 0, stream>>>(
        n, pos3d, scale3d, reinterpret_cast<const float4 *>(quat), vol[0],
        vol[1], vol[2], world[0], world[1], world[2],
        reinterpret_cast<const float4 *>(pos_radii_grad),
        reinterpret_cast<const float2 *>(conics_grad),
        reinterpret_cast<const float4 *>(pos_radii), pos_grad, scale_grad,
        reinterpret_cast<float4 *>(quat_grad));
    count_launches(1);
    return cudaGetLastError();
}

}  // namespace gsv
