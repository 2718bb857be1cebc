/*
 * gsv_oracle.c - CPU restatement of the reference's Gaussian voxelization
 * path, used ONLY as test infrastructure: the parity tests, smoke() and
 * bench.py's cpu_baseline leg call it as the checker. The product path
 * (gs_voxelizer_b200) never calls it.
 *
 * Each function cites the reference code it restates (PaPieta/gs-voxelizer,
 * paths relative to the project root). Arithmetic is IEEE float32, evaluated
 * in source order (built with -ffp-contract=off). The reference's GPU build
 * uses --use_fast_math (approximate division, sqrt, log, exp; fused
 * multiply-adds), so float outputs agree to a few ulp, and integer tile
 * bounds agree except where the truncated value lies within a few ulp of an
 * integer; oracle_project_fwd reports those pre-truncation values so the
 * tests can tell such boundary cases apart.
 *
 * OpenMP parallel loops keep results deterministic: every output element is
 * written by one thread, in a fixed summation order.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define TILE 8
#define TILE_VOX (TILE * TILE * TILE)

typedef struct {
    float m[3][3]; /* column-major: m[col][row], GLM convention */
} mat3;

static mat3 mat3_mul(mat3 a, mat3 b) {
    mat3 o;
    for (int c = 0; c < 3; ++c)
        for (int r = 0; r < 3; ++r)
            o.m[c][r] = a.m[0][r] * b.m[c][0] + a.m[1][r] * b.m[c][1] +
                        a.m[2][r] * b.m[c][2];
    return o;
}

static mat3 mat3_t(mat3 a) {
    mat3 o;
    for (int c = 0; c < 3; ++c)
        for (int r = 0; r < 3; ++r) o.m[c][r] = a.m[r][c];
    return o;
}

static mat3 mat3_diag(float a, float b, float c) {
    mat3 o;
    memset(&o, 0, sizeof(o));
    o.m[0][0] = a;
    o.m[1][1] = b;
    o.m[2][2] = c;
    return o;
}

/* optim_to_render_helpers.cuh:15-37 - quaternion (w,x,y,z) stored in a
 * float4's (x,y,z,w) slots, normalised, to a column-major rotation. */
static mat3 quat_to_rot(const float *q4, float *wxyz_out) {
    const float qx = q4[0], qy = q4[1], qz = q4[2], qw = q4[3];
    const float s = 1.0f / sqrtf(qw * qw + qx * qx + qy * qy + qz * qz);
    const float w = qx * s, x = qy * s, y = qz * s, z = qw * s;
    if (wxyz_out) {
        wxyz_out[0] = w;
        wxyz_out[1] = x;
        wxyz_out[2] = y;
        wxyz_out[3] = z;
    }
    mat3 R;
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

/* CUDA's float->int conversion saturates and maps NaN to 0. */
static int f2i_trunc(float v) {
    if (v != v) return 0;
    if (v >= 2147483647.0f) return 2147483647;
    if (v <= -2147483648.0f) return (-2147483647 - 1);
    return (int)v;
}

static int imin(int a, int b) { return a < b ? a : b; }
static int imax(int a, int b) { return a > b ? a : b; }

/* voxel-space covariance, optim_to_render.cu:84-103 */
static mat3 voxel_cov(const float *s3, mat3 R, float vox_x, float vox_y,
                      float vox_z, mat3 *M2_out) {
    mat3 S = mat3_diag(s3[0], s3[1], s3[2]);
    mat3 M = mat3_mul(S, R);
    mat3 cov = mat3_mul(mat3_t(M), M);
    mat3 M2 = mat3_diag(1.f / vox_x, 1.f / vox_y, 1.f / vox_z);
    if (M2_out) *M2_out = M2;
    return mat3_mul(mat3_mul(mat3_t(M2), cov), M2);
}

/*
 * optim_to_render.cu:48-172 (kernel) with bindings.cu:44-189 (axis mapping:
 * vol = (Z, Y, X), world / center tuples in (z, y, x) order).
 * bounds_f (optional, [n,6]) receives the six pre-truncation tile values
 * (lo.x, lo.y, lo.z, hi.x, hi.y, hi.z) divided by the tile size.
 */
void oracle_project_fwd(int n, int C, const float *pos3d, const float *scale3d,
                        const float *quat, const float *intens,
                        const int *vol, const float *world,
                        const float *center, float *pos_radii, float *conics,
                        int *tmin, int *tmax, int *ntiles, float *bounds_f) {
    const int Z = vol[0], Y = vol[1], X = vol[2];
    const int Tx = (X + TILE - 1) / TILE, Ty = (Y + TILE - 1) / TILE,
              Tz = (Z + TILE - 1) / TILE;
    const float vox_z = world[0] / (float)Z, vox_y = world[1] / (float)Y,
                vox_x = world[2] / (float)X;
#pragma omp parallel for schedule(static)
    for (int i = 0; i < n; ++i) {
        float *pr = pos_radii + 4 * i;
        float *cq = conics + 6 * i;
        int *lo = tmin + 3 * i, *hi = tmax + 3 * i;
        memset(pr, 0, 4 * sizeof(float));
        memset(cq, 0, 6 * sizeof(float));
        lo[0] = lo[1] = lo[2] = hi[0] = hi[1] = hi[2] = 0;
        ntiles[i] = 0;
        if (bounds_f)
            for (int k = 0; k < 6; ++k) bounds_f[6 * i + k] = 0.f;

        const float *p = pos3d + 3 * i, *s = scale3d + 3 * i;
        const float px = (p[0] - center[2] + (world[2] * 0.5f)) / vox_x;
        const float py = (p[1] - center[1] + (world[1] * 0.5f)) / vox_y;
        const float pz = (p[2] - center[0] + (world[0] * 0.5f)) / vox_z;
        const mat3 R = quat_to_rot(quat + 4 * i, NULL);
        const mat3 cov = voxel_cov(s, R, vox_x, vox_y, vox_z, NULL);
        const float a = cov.m[0][0], b = cov.m[0][1], c = cov.m[0][2];
        const float d = cov.m[1][1], e = cov.m[1][2], f = cov.m[2][2];
        const float det =
            a * d * f + 2 * b * c * e - a * e * e - f * b * b - d * c * c;
        if (det == 0.0f) continue;
        const float inv_det = 1.0f / det;
        const float q[6] = {
            inv_det * (d * f - e * e), inv_det * (c * e - b * f),
            inv_det * (b * e - c * d), inv_det * (a * f - c * c),
            inv_det * (b * c - a * e), inv_det * (a * d - b * b)};
        const float smax = fmaxf(s[0], fmaxf(s[1], s[2]));
        const float radius =
            ceilf((3.f * smax) / fminf(vox_x, fminf(vox_y, vox_z)));
        float mean = 0.f;
        for (int k = 0; k < C; ++k) mean += intens[i * C + k];
        mean /= (float)C;
        const float lthr = logf(mean * (1 / 0.000001f));
        const float extent = fminf(3.f, sqrtf(2.0f * lthr));
        const float r3[3] = {fmaxf(0.0f, (sqrtf(a) * extent) - 0.5f),
                             fmaxf(0.0f, (sqrtf(d) * extent) - 0.5f),
                             fmaxf(0.0f, (sqrtf(f) * extent) - 0.5f)};
        if (radius <= 0.f || px + radius < 0.f || px - radius > (float)X ||
            py + radius < 0.f || py - radius > (float)Y ||
            pz + radius < 0.f || pz - radius > (float)Z)
            continue;
        /* get_tile_bbox, optim_to_render.cu:26-40 */
        const float ctr[3] = {px, py, pz};
        const int bound[3] = {Tx, Ty, Tz};
        int l[3], h[3];
        float lf[3], hf[3];
        for (int k = 0; k < 3; ++k) {
            lf[k] = (ctr[k] - r3[k]) / (float)TILE;
            hf[k] = (ctr[k] + r3[k] + (float)(TILE - 1)) / (float)TILE;
            l[k] = imin(bound[k], imax(0, f2i_trunc(lf[k])));
            h[k] = imin(bound[k], imax(0, f2i_trunc(hf[k])));
        }
        const int tv = (h[0] - l[0]) * (h[1] - l[1]) * (h[2] - l[2]);
        if (bounds_f)
            for (int k = 0; k < 3; ++k) {
                bounds_f[6 * i + k] = lf[k];
                bounds_f[6 * i + 3 + k] = hf[k];
            }
        if (tv <= 0) continue;
        pr[0] = px;
        pr[1] = py;
        pr[2] = pz;
        pr[3] = radius;
        for (int k = 0; k < 6; ++k) cq[k] = q[k];
        for (int k = 0; k < 3; ++k) {
            lo[k] = l[k];
            hi[k] = h[k];
        }
        ntiles[i] = tv;
    }
}

/* optim_to_render.cu:186-239 */
static mat3 cov_grad(mat3 cov, mat3 M2, const float *g) {
    const float a = cov.m[0][0], b = cov.m[0][1], c = cov.m[0][2];
    const float d = cov.m[1][1], e = cov.m[1][2], f = cov.m[2][2];
    const float det =
        a * d * f + 2 * b * c * e - a * e * e - f * b * b - d * c * c;
    const float k = 1.0f / ((det * det) + 0.0000001f);
    mat3 out;
    memset(&out, 0, sizeof(out));
    if (k == 0) return out;
    const float da = d * f - e * e, db = 2 * c * e - 2 * f * b,
                dc = 2 * b * e - 2 * d * c, dd = a * f - c * c,
                de = 2 * b * c - 2 * a * e, df = a * d - b * b;
    const float nb = c * e - b * f, nc = b * e - c * d, ne = b * c - a * e;
    const float g0 = g[0], g1 = g[1], g2 = g[2], g3 = g[3], g4 = g[4],
                g5 = g[5];
    const float ga = k * (-da * da * g0 - nb * da * g1 - nc * da * g2 +
                          (f * det - dd * da) * g3 + (-e * det - ne * da) * g4 +
                          (d * det - df * da) * g5);
    const float gb = k * (-da * db * g0 + (-f * det - nb * db) * g1 +
                          (e * det - nc * db) * g2 - dd * db * g3 +
                          (c * det - ne * db) * g4 +
                          (-2 * b * det - df * db) * g5);
    const float gc = k * (-da * dc * g0 + (e * det - nb * dc) * g1 +
                          (-d * det - nc * dc) * g2 +
                          (-2 * c * det - dd * dc) * g3 +
                          (b * det - ne * dc) * g4 - df * dc * g5);
    const float gd = k * ((f * det - da * dd) * g0 - nb * dd * g1 +
                          (-c * det - nc * dd) * g2 - dd * dd * g3 -
                          ne * dd * g4 + (a * det - df * dd) * g5);
    const float ge = k * ((-2 * e * det - da * de) * g0 +
                          (c * det - nb * de) * g1 + (b * det - nc * de) * g2 -
                          dd * de * g3 + (-a * det - ne * de) * g4 +
                          -df * de * g5);
    const float gf = k * ((d * det - da * df) * g0 + (-b * det - nb * df) * g1 -
                          nc * df * g2 + (a * det - dd * df) * g3 -
                          ne * df * g4 - df * df * g5);
    mat3 G;
    G.m[0][0] = ga; G.m[0][1] = gb; G.m[0][2] = gc;
    G.m[1][0] = gb; G.m[1][1] = gd; G.m[1][2] = ge;
    G.m[2][0] = gc; G.m[2][1] = ge; G.m[2][2] = gf;
    mat3 W = mat3_mul(mat3_mul(M2, G), mat3_t(M2));
    mat3 Wt = mat3_t(W);
    for (int cc = 0; cc < 3; ++cc)
        for (int r = 0; r < 3; ++r)
            out.m[cc][r] = 0.5f * (W.m[cc][r] + Wt.m[cc][r]);
    return out;
}

/* optim_to_render.cu:246-336 and optim_to_render_helpers.cuh:51-75 */
void oracle_project_bwd(int n, const float *pos3d, const float *scale3d,
                        const float *quat, const int *vol, const float *world,
                        const float *pos_radii_grad, const float *conics_grad,
                        const float *pos_radii, float *pos_grad,
                        float *scale_grad, float *quat_grad) {
    (void)pos3d;
    const int Z = vol[0], Y = vol[1], X = vol[2];
    const float vox_z = world[0] / (float)Z, vox_y = world[1] / (float)Y,
                vox_x = world[2] / (float)X;
#pragma omp parallel for schedule(static)
    for (int i = 0; i < n; ++i) {
        float *gp = pos_grad + 3 * i, *gs = scale_grad + 3 * i,
              *gq = quat_grad + 4 * i;
        memset(gp, 0, 3 * sizeof(float));
        memset(gs, 0, 3 * sizeof(float));
        memset(gq, 0, 4 * sizeof(float));
        if (!(pos_radii[4 * i + 3] > 0)) continue;
        const float *s = scale3d + 3 * i;
        float wxyz[4];
        const mat3 R = quat_to_rot(quat + 4 * i, wxyz);
        mat3 M2;
        const mat3 cov = voxel_cov(s, R, vox_x, vox_y, vox_z, &M2);
        const mat3 cg = cov_grad(cov, M2, conics_grad + 6 * i);
        mat3 dS;
        for (int c = 0; c < 3; ++c)
            for (int r = 0; r < 3; ++r)
                dS.m[c][r] = (c == r) ? cg.m[c][r] : 0.5f * cg.m[c][r];
        mat3 S2 = mat3_diag(2.0f * s[0], 2.0f * s[1], 2.0f * s[2]);
        const mat3 Rg = mat3_mul(mat3_mul(S2, R), dS);
        mat3 v = mat3_t(Rg);
        const mat3 Rt = mat3_t(R);
        for (int k = 0; k < 3; ++k)
            gs[k] = Rt.m[k][0] * v.m[k][0] + Rt.m[k][1] * v.m[k][1] +
                    Rt.m[k][2] * v.m[k][2];
        for (int k = 0; k < 3; ++k)
            for (int r = 0; r < 3; ++r) v.m[k][r] *= s[k];
        /* reference quirk: position gradient multiplied by voxel size */
        gp[0] = pos_radii_grad[4 * i + 0] * vox_x;
        gp[1] = pos_radii_grad[4 * i + 1] * vox_y;
        gp[2] = pos_radii_grad[4 * i + 2] * vox_z;
        const float w = wxyz[0], x = wxyz[1], y = wxyz[2], z = wxyz[3];
        gq[0] = 2 * z * (v.m[0][1] - v.m[1][0]) +
                2 * y * (v.m[2][0] - v.m[0][2]) +
                2 * x * (v.m[1][2] - v.m[2][1]);
        gq[1] = 2 * y * (v.m[1][0] + v.m[0][1]) +
                2 * z * (v.m[2][0] + v.m[0][2]) +
                2 * w * (v.m[1][2] - v.m[2][1]) -
                4 * x * (v.m[2][2] + v.m[1][1]);
        gq[2] = 2 * x * (v.m[1][0] + v.m[0][1]) +
                2 * w * (v.m[2][0] - v.m[0][2]) +
                2 * z * (v.m[1][2] + v.m[2][1]) -
                4 * y * (v.m[2][2] + v.m[0][0]);
        gq[3] = 2 * w * (v.m[0][1] - v.m[1][0]) +
                2 * x * (v.m[2][0] + v.m[0][2]) +
                2 * y * (v.m[1][2] + v.m[2][1]) -
                4 * z * (v.m[1][1] + v.m[0][0]);
    }
}

/*
 * bin_and_sort_gaussians.cu:11-62 + bindings.cu:261-360: pairs emitted per
 * Gaussian in gaussian order (z, y, x nested), stably sorted by tile id;
 * tile_bins [T,2] gets [start, end) for tiles that occur, (0,0) otherwise.
 * Restated as a stable counting sort. Tiles restricted to [tz0, tz1) with
 * slab-local ids (tz1 < 0 = whole volume). Returns the pair count; with
 * ids_out == NULL only tile_bins is written. Returns -1 (and writes no ids)
 * if the count differs from `capacity`.
 */
int64_t oracle_bin(int n, const int *tmin, const int *tmax, const int *vol,
                   int tz0, int tz1, int *ids_out, int *bins_out,
                   int64_t capacity) {
    const int Z = vol[0], Y = vol[1], X = vol[2];
    const int Tx = (X + TILE - 1) / TILE, Ty = (Y + TILE - 1) / TILE,
              Tz = (Z + TILE - 1) / TILE;
    if (tz1 < 0) tz1 = Tz;
    const int64_t T = (int64_t)(tz1 - tz0) * Ty * Tx;
    int64_t *count = (int64_t *)calloc((size_t)T + 1, sizeof(int64_t));
    int64_t total = 0;
    for (int i = 0; i < n; ++i) {
        const int z0 = imax(tmin[3 * i + 2], tz0), z1 = imin(tmax[3 * i + 2], tz1);
        for (int z = z0; z < z1; ++z)
            for (int y = tmin[3 * i + 1]; y < tmax[3 * i + 1]; ++y)
                for (int x = tmin[3 * i + 0]; x < tmax[3 * i + 0]; ++x) {
                    count[((int64_t)(z - tz0) * Ty + y) * Tx + x]++;
                    total++;
                }
    }
    int64_t run = 0;
    for (int64_t t = 0; t < T; ++t) {
        const int64_t c = count[t];
        bins_out[2 * t] = c ? (int)run : 0;
        bins_out[2 * t + 1] = c ? (int)(run + c) : 0;
        count[t] = run;
        run += c;
    }
    if (!ids_out) {
        free(count);
        return total;
    }
    if (total != capacity) {
        free(count);
        return -1;
    }
    for (int i = 0; i < n; ++i) {
        const int z0 = imax(tmin[3 * i + 2], tz0), z1 = imin(tmax[3 * i + 2], tz1);
        for (int z = z0; z < z1; ++z)
            for (int y = tmin[3 * i + 1]; y < tmax[3 * i + 1]; ++y)
                for (int x = tmin[3 * i + 0]; x < tmax[3 * i + 0]; ++x)
                    ids_out[count[((int64_t)(z - tz0) * Ty + y) * Tx + x]++] = i;
    }
    free(count);
    return total;
}

/* sigma of voxelize.cu:125-131 */
static inline float vox_sigma(const float *q, float dx, float dy, float dz) {
    return -0.5f * (q[0] * dx * dx + q[3] * dy * dy + q[5] * dz * dz) -
           (q[1] * dx * dy + q[2] * dx * dz + q[4] * dy * dz);
}

/* voxelize.cu:39-164 with bindings.cu:362-457: one output per voxel, the
 * tile's Gaussians accumulated in sorted-list order. Slab-restricted like
 * oracle_bin (out covers voxel z in [8*tz0, min(Z, 8*tz1))). */
void oracle_vox_fwd(const int *vol, int tz0, int tz1, int C, const int *ids,
                    const int *bins, const float *pos_radii,
                    const float *conics, const float *intens, float *out) {
    const int Z = vol[0], Y = vol[1], X = vol[2];
    const int Tx = (X + TILE - 1) / TILE, Ty = (Y + TILE - 1) / TILE,
              Tz = (Z + TILE - 1) / TILE;
    if (tz1 < 0) tz1 = Tz;
    const int zb = tz0 * TILE, ze = imin(Z, tz1 * TILE);
    const int64_t T = (int64_t)(tz1 - tz0) * Ty * Tx;
#pragma omp parallel for schedule(dynamic, 16)
    for (int64_t t = 0; t < T; ++t) {
        const int tx = (int)(t % Tx), ty = (int)((t / Tx) % Ty),
                  tz = (int)(t / ((int64_t)Tx * Ty)) + tz0;
        const int b0 = bins[2 * t], b1 = bins[2 * t + 1];
        for (int lz = 0; lz < TILE; ++lz)
            for (int ly = 0; ly < TILE; ++ly)
                for (int lx = 0; lx < TILE; ++lx) {
                    const int x = tx * TILE + lx, y = ty * TILE + ly,
                              z = tz * TILE + lz;
                    if (x >= X || y >= Y || z >= ze) continue;
                    const float vx = (float)x + 0.5f, vy = (float)y + 0.5f,
                                vz = (float)z + 0.5f;
                    float acc[4] = {0.f, 0.f, 0.f, 0.f};
                    for (int k = b0; k < b1; ++k) {
                        const int g = ids[k];
                        const float *p = pos_radii + 4 * g;
                        const float *q = conics + 6 * g;
                        const float s = vox_sigma(q, p[0] - vx, p[1] - vy,
                                                  p[2] - vz);
                        if (s > 0.f || isnan(s) || isinf(s)) continue;
                        const float alpha = expf(s);
                        float mean = 0.f;
                        for (int c = 0; c < C; ++c) mean += intens[C * g + c];
                        mean /= (float)C;
                        if (alpha * mean < 0.000001f) continue;
                        for (int c = 0; c < C; ++c)
                            acc[c] += intens[C * g + c] * alpha;
                    }
                    const int64_t o =
                        (((int64_t)(z - zb) * Y + y) * X + x) * C;
                    for (int c = 0; c < C; ++c) out[o + c] = acc[c];
                }
    }
}

/*
 * voxelize.cu:368-574 (per-Gaussian backward; the per-voxel variant at
 * :170-366 computes the same sums in another order): for every (Gaussian,
 * tile) pair the tile's voxels are visited in z, y, x order and the
 * gradient terms accumulated in float; the pair totals are then added to the
 * Gaussian's gradients in tile order. Parallel over Gaussians (each thread
 * owns its Gaussian's outputs), so the result is deterministic.
 * pos_grad is [n,4] (w = 0), conic_grad [n,6], int_grad [n,C].
 */
void oracle_vox_bwd(const int *vol, int tz0, int tz1, int C, int n,
                    const int *tmin, const int *tmax, const float *pos_radii,
                    const float *conics, const float *intens,
                    const float *grad, float *pos_grad, float *conic_grad,
                    float *int_grad) {
    const int Z = vol[0], Y = vol[1], X = vol[2];
    const int Tz = (Z + TILE - 1) / TILE;
    if (tz1 < 0) tz1 = Tz;
    const int zb = tz0 * TILE, ze = imin(Z, tz1 * TILE);
#pragma omp parallel for schedule(dynamic, 64)
    for (int g = 0; g < n; ++g) {
        float gp[3] = {0, 0, 0}, gc[6] = {0, 0, 0, 0, 0, 0},
              gi[4] = {0, 0, 0, 0};
        const float *p = pos_radii + 4 * g;
        const float *q = conics + 6 * g;
        const float *I = intens + C * g;
        float mean = 0.f;
        for (int c = 0; c < C; ++c) mean += I[c];
        mean /= (float)C;
        const int z0 = imax(tmin[3 * g + 2], tz0), z1 = imin(tmax[3 * g + 2], tz1);
        for (int tz = z0; tz < z1; ++tz)
            for (int ty = tmin[3 * g + 1]; ty < tmax[3 * g + 1]; ++ty)
                for (int tx = tmin[3 * g + 0]; tx < tmax[3 * g + 0]; ++tx) {
                    float lp[3] = {0, 0, 0}, lc[6] = {0, 0, 0, 0, 0, 0},
                          li[4] = {0, 0, 0, 0};
                    for (int v = 0; v < TILE_VOX; ++v) {
                        const int x = tx * TILE + (v % TILE);
                        const int y = ty * TILE + (v / TILE) % TILE;
                        const int z = tz * TILE + v / (TILE * TILE);
                        if (x >= X || y >= Y || z >= ze) continue;
                        const float dx = p[0] - ((float)x + 0.5f);
                        const float dy = p[1] - ((float)y + 0.5f);
                        const float dz = p[2] - ((float)z + 0.5f);
                        const float s = vox_sigma(q, dx, dy, dz);
                        if (s > 0.f || isnan(s) || isinf(s)) continue;
                        const float d = expf(s);
                        if (d * mean < 0.000001f) continue;
                        const float *gv =
                            grad + (((int64_t)(z - zb) * Y + y) * X + x) * C;
                        float sg = 0.f;
                        for (int c = 0; c < C; ++c) {
                            li[c] += d * gv[c];
                            sg += I[c] * gv[c];
                        }
                        sg *= d;
                        lc[0] += -0.5f * sg * dx * dx;
                        lc[1] += -sg * dx * dy;
                        lc[2] += -sg * dx * dz;
                        lc[3] += -0.5f * sg * dy * dy;
                        lc[4] += -sg * dy * dz;
                        lc[5] += -0.5f * sg * dz * dz;
                        lp[0] += -sg * (q[0] * dx + q[1] * dy + q[2] * dz);
                        lp[1] += -sg * (q[1] * dx + q[3] * dy + q[4] * dz);
                        lp[2] += -sg * (q[2] * dx + q[4] * dy + q[5] * dz);
                    }
                    for (int k = 0; k < 3; ++k) gp[k] += lp[k];
                    for (int k = 0; k < 6; ++k) gc[k] += lc[k];
                    for (int c = 0; c < C; ++c) gi[c] += li[c];
                }
        pos_grad[4 * g + 0] = gp[0];
        pos_grad[4 * g + 1] = gp[1];
        pos_grad[4 * g + 2] = gp[2];
        pos_grad[4 * g + 3] = 0.f;
        for (int k = 0; k < 6; ++k) conic_grad[6 * g + k] = gc[k];
        for (int c = 0; c < C; ++c) int_grad[C * g + c] = gi[c];
    }
}

/* L1 loss and its gradient as the bench's training step uses them
 * (torch.nn.functional.l1_loss, mean reduction): returns sum|v - t| / V and
 * writes dL/dvol = sign(v - t) / V. */
double oracle_l1(int64_t nvox, const float *v, const float *t, double denom,
                 float *grad) {
    double s = 0.0;
#pragma omp parallel for reduction(+ : s) schedule(static)
    for (int64_t i = 0; i < nvox; ++i) {
        const float d = v[i] - t[i];
        s += fabs((double)d);
        if (grad)
            grad[i] = (d > 0.f ? 1.f : (d < 0.f ? -1.f : 0.f)) / (float)denom;
    }
    return s / denom;
}

/* ------------------------------------------------------------------ SSIM
 * 3D SSIM (Wang, Bovik, Sheikh, Simoncelli 2004) as the reference's tests
 * use it through the external fused_ssim3d (test/test_gs_voxelizer.py:62):
 * the mean over all voxels and channels of
 *   S = (2 mu_x mu_y + C1)(2 s_xy + C2) / ((mu_x^2 + mu_y^2 + C1)(s_x^2 + s_y^2 + C2))
 * with local statistics under the separable window w (11 taps), zero
 * padding. Restated from the paper's definition (the fused_ssim sources
 * are not part of the reference); float64 throughout. grad (nullable) =
 * d mean(S) / d img1.
 * Volumes are planar [nch][D][H][W].
 */
static void blur3(int D, int H, int W, const double *w, int R, const double *in,
                  double *out, double *tmp) {
    const size_t plane = (size_t)H * W;
    /* x */
#pragma omp parallel for
    for (long long zy = 0; zy < (long long)D * H; ++zy)
        for (int x = 0; x < W; ++x) {
            double acc = 0.0;
            for (int k = -R; k <= R; ++k)
                if (x + k >= 0 && x + k < W) acc += w[k + R] * in[zy * W + x + k];
            out[zy * W + x] = acc;
        }
    /* y */
#pragma omp parallel for
    for (long long z = 0; z < D; ++z)
        for (int y = 0; y < H; ++y)
            for (int x = 0; x < W; ++x) {
                double acc = 0.0;
                for (int k = -R; k <= R; ++k)
                    if (y + k >= 0 && y + k < H)
                        acc += w[k + R] * out[z * plane + (size_t)(y + k) * W + x];
                tmp[z * plane + (size_t)y * W + x] = acc;
            }
    /* z */
#pragma omp parallel for
    for (long long z = 0; z < D; ++z)
        for (size_t q = 0; q < plane; ++q) {
            double acc = 0.0;
            for (int k = -R; k <= R; ++k)
                if (z + k >= 0 && z + k < D) acc += w[k + R] * tmp[(z + k) * plane + q];
            out[z * plane + q] = acc;
        }
}

double oracle_ssim3d(int nch, int D, int H, int W, const float *a, const float *b,
                     double C1, double C2, const double *w, int R, float *grad) {
    const size_t nv = (size_t)D * H * W;
    const double inv_n = 1.0 / ((double)nv * nch);
    double *in = malloc(sizeof(double) * nv), *tmp = malloc(sizeof(double) * nv);
    double *m[5];
    for (int k = 0; k < 5; ++k) m[k] = malloc(sizeof(double) * nv);
    double total = 0.0;
    for (int c = 0; c < nch; ++c) {
        const float *x = a + c * nv, *y = b + c * nv;
        for (int k = 0; k < 5; ++k) {
            for (size_t i = 0; i < nv; ++i) {
                const double xv = x[i], yv = y[i];
                in[i] = k == 0 ? xv : k == 1 ? yv : k == 2 ? xv * xv
                      : k == 3 ? yv * yv : xv * yv;
            }
            blur3(D, H, W, w, R, in, m[k], tmp);
        }
        /* S and the three G maps (for d mean / d S = 1/N) in m[2..4] */
        double part = 0.0;
        for (size_t i = 0; i < nv; ++i) {
            const double mx = m[0][i], my = m[1][i];
            const double sxx = m[2][i] - mx * mx, syy = m[3][i] - my * my,
                         sxy = m[4][i] - mx * my;
            const double A1 = 2 * mx * my + C1, A2 = 2 * sxy + C2;
            const double B1 = mx * mx + my * my + C1, B2 = sxx + syy + C2;
            const double S = A1 * A2 / (B1 * B2);
            part += S;
            m[2][i] = inv_n * (2 * my * (A2 - A1) / (B1 * B2) +
                               2 * mx * S * (1.0 / B2 - 1.0 / B1));
            m[3][i] = inv_n * (-S / B2);
            m[4][i] = inv_n * (2 * A1 / (B1 * B2));
        }
        total += part;
        if (grad) {
            float *g = grad + c * nv;
            blur3(D, H, W, w, R, m[2], m[0], tmp);
            blur3(D, H, W, w, R, m[3], m[1], tmp);
            blur3(D, H, W, w, R, m[4], m[2], tmp);
            for (size_t i = 0; i < nv; ++i)
                g[i] = (float)(m[0][i] + 2.0 * x[i] * m[1][i] + y[i] * m[2][i]);
        }
    }
    free(in);
    free(tmp);
    for (int k = 0; k < 5; ++k) free(m[k]);
    return total * inv_n;
}

/* -------------------------------------------------------------------- TV
 * 3D total variation (Rudin, Osher, Fatemi 1992) with forward differences
 * d_a(v) = x(v + e_a) - x(v) inside the volume (0 across the far edge):
 * iso: mean sqrt(dx^2 + dy^2 + dz^2 + eps); else mean (|dx| + |dy| + |dz|).
 * The companion external package (fused-3D-tv) is not part of the
 * reference; restated from the definition, float64. grad (nullable) =
 * d TV / d x. Planar [nch][D][H][W].
 */
static void tv_diff(const float *x, int D, int H, int W, int z, int y, int xx,
                    double *d) {
    const size_t i = ((size_t)z * H + y) * W + xx;
    d[0] = xx + 1 < W ? (double)x[i + 1] - x[i] : 0.0;
    d[1] = y + 1 < H ? (double)x[i + W] - x[i] : 0.0;
    d[2] = z + 1 < D ? (double)x[i + (size_t)H * W] - x[i] : 0.0;
}

static double tv_term(const double *d, int iso, double eps) {
    return iso ? sqrt(d[0] * d[0] + d[1] * d[1] + d[2] * d[2] + eps)
               : fabs(d[0]) + fabs(d[1]) + fabs(d[2]);
}

static double sgn(double v) { return (v > 0) - (v < 0); }

double oracle_tv3d(int nch, int D, int H, int W, const float *xs, int iso,
                   double eps, float *grad) {
    const size_t nv = (size_t)D * H * W;
    const double inv_n = 1.0 / ((double)nv * nch);
    double total = 0.0;
    for (int c = 0; c < nch; ++c) {
        const float *x = xs + c * nv;
        double part = 0.0;
#pragma omp parallel for reduction(+ : part)
        for (long long z = 0; z < D; ++z)
            for (int y = 0; y < H; ++y)
                for (int xx = 0; xx < W; ++xx) {
                    double d[3];
                    tv_diff(x, D, H, W, (int)z, y, xx, d);
                    const double t = tv_term(d, iso, eps);
                    part += t;
                    if (!grad) continue;
                    double g = iso ? -(d[0] + d[1] + d[2]) / t
                                   : -(sgn(d[0]) + sgn(d[1]) + sgn(d[2]));
                    const int nz[3][3] = {{0, 0, -1}, {0, -1, 0}, {-1, 0, 0}};
                    for (int a = 0; a < 3; ++a) {  /* neighbours behind v */
                        const int zz = (int)z + nz[a][0], yy = y + nz[a][1],
                                  xw = xx + nz[a][2];
                        if (zz < 0 || yy < 0 || xw < 0) continue;
                        double e[3];
                        tv_diff(x, D, H, W, zz, yy, xw, e);
                        g += iso ? e[a] / tv_term(e, 1, eps) : sgn(e[a]);
                    }
                    grad[c * nv + ((size_t)z * H + y) * W + xx] = (float)(g * inv_n);
                }
        total += part;
    }
    return total * inv_n;
}

int oracle_num_threads(void) {
#ifdef _OPENMP
    extern int omp_get_max_threads(void);
    return omp_get_max_threads();
#else
    return 1;
#endif
}
