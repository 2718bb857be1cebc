// Minimal stand-in for the GLM 1.0.3 headers the reference includes
// (gs_voxelizer/cuda/optim_to_render*.cu[h]); GLM itself is not installed
// here and there is no network to fetch it. Written from GLM's documented
// semantics, covering only what the reference uses:
//   mat3 is column-major (m[c] is column c, m[c][r] row r of it);
//   mat3(s) is s on the diagonal; mat3(9 scalars) fills column by column;
//   (A * B)[c][r] = A[0][r]*B[c][0] + A[1][r]*B[c][1] + A[2][r]*B[c][2];
//   scalar * mat3, mat3 + mat3, transpose(mat3), dot(vec3, vec3),
//   vec3 *= scalar.
// Used only to compile the reference for the parity oracle in oracle/_ref.
#pragma once

#if defined(__CUDACC__)
#define GLM_SHIM_FN __host__ __device__ inline
#else
#define GLM_SHIM_FN inline
#endif

namespace glm {

struct vec3 {
    float x, y, z;
    GLM_SHIM_FN vec3() : x(0.f), y(0.f), z(0.f) {}
    GLM_SHIM_FN vec3(float a, float b, float c) : x(a), y(b), z(c) {}
    GLM_SHIM_FN float &operator[](int i) { return i == 0 ? x : (i == 1 ? y : z); }
    GLM_SHIM_FN const float &operator[](int i) const {
        return i == 0 ? x : (i == 1 ? y : z);
    }
    GLM_SHIM_FN vec3 &operator*=(float s) {
        x *= s;
        y *= s;
        z *= s;
        return *this;
    }
};

GLM_SHIM_FN float dot(const vec3 &a, const vec3 &b) {
    return a.x * b.x + a.y * b.y + a.z * b.z;
}

struct mat3 {
    vec3 col[3];
    GLM_SHIM_FN mat3() : mat3(1.f) {}
    GLM_SHIM_FN explicit mat3(float s) {
        col[0] = vec3(s, 0.f, 0.f);
        col[1] = vec3(0.f, s, 0.f);
        col[2] = vec3(0.f, 0.f, s);
    }
    GLM_SHIM_FN mat3(float x0, float y0, float z0, float x1, float y1, float z1,
                     float x2, float y2, float z2) {
        col[0] = vec3(x0, y0, z0);
        col[1] = vec3(x1, y1, z1);
        col[2] = vec3(x2, y2, z2);
    }
    GLM_SHIM_FN vec3 &operator[](int c) { return col[c]; }
    GLM_SHIM_FN const vec3 &operator[](int c) const { return col[c]; }
};

GLM_SHIM_FN mat3 operator*(const mat3 &a, const mat3 &b) {
    mat3 o(0.f);
    for (int c = 0; c < 3; ++c)
        for (int r = 0; r < 3; ++r)
            o[c][r] = a[0][r] * b[c][0] + a[1][r] * b[c][1] + a[2][r] * b[c][2];
    return o;
}

GLM_SHIM_FN mat3 operator*(float s, const mat3 &a) {
    mat3 o(0.f);
    for (int c = 0; c < 3; ++c)
        for (int r = 0; r < 3; ++r) o[c][r] = s * a[c][r];
    return o;
}

GLM_SHIM_FN mat3 operator+(const mat3 &a, const mat3 &b) {
    mat3 o(0.f);
    for (int c = 0; c < 3; ++c)
        for (int r = 0; r < 3; ++r) o[c][r] = a[c][r] + b[c][r];
    return o;
}

GLM_SHIM_FN mat3 transpose(const mat3 &a) {
    mat3 o(0.f);
    for (int c = 0; c < 3; ++c)
        for (int r = 0; r < 3; ++r) o[c][r] = a[r][c];
    return o;
}

}  // namespace glm
