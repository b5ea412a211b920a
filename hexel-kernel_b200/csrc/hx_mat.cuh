// Minimal column-major 2x2 / 3x3 float matrices for the projection math.
//
// Storage and product order follow the column-major convention the
// reference's math is written in (m[col][row]; each product entry summed over
// the inner index in increasing order).  Keeping the same summation order
// keeps the same floating-point rounding, which the bit-exact tile counts of
// the projection kernels depend on.
#pragma once

namespace hx {

struct Mat2 {
    float m[2][2];  // m[col][row]
};

__device__ __forceinline__ Mat2 mat2_diag(float d) {
    Mat2 r;
    r.m[0][0] = d; r.m[0][1] = 0.f;
    r.m[1][0] = 0.f; r.m[1][1] = d;
    return r;
}

__device__ __forceinline__ Mat2 mat2(float c0r0, float c0r1, float c1r0, float c1r1) {
    Mat2 r;
    r.m[0][0] = c0r0; r.m[0][1] = c0r1;
    r.m[1][0] = c1r0; r.m[1][1] = c1r1;
    return r;
}

__device__ __forceinline__ Mat2 mul(const Mat2& a, const Mat2& b) {
    Mat2 r;
    r.m[0][0] = a.m[0][0] * b.m[0][0] + a.m[1][0] * b.m[0][1];
    r.m[0][1] = a.m[0][1] * b.m[0][0] + a.m[1][1] * b.m[0][1];
    r.m[1][0] = a.m[0][0] * b.m[1][0] + a.m[1][0] * b.m[1][1];
    r.m[1][1] = a.m[0][1] * b.m[1][0] + a.m[1][1] * b.m[1][1];
    return r;
}

__device__ __forceinline__ Mat2 transpose(const Mat2& a) {
    return mat2(a.m[0][0], a.m[1][0], a.m[0][1], a.m[1][1]);
}

__device__ __forceinline__ Mat2 neg(const Mat2& a) {
    return mat2(-a.m[0][0], -a.m[0][1], -a.m[1][0], -a.m[1][1]);
}

__device__ __forceinline__ Mat2 add(const Mat2& a, const Mat2& b) {
    return mat2(a.m[0][0] + b.m[0][0], a.m[0][1] + b.m[0][1], a.m[1][0] + b.m[1][0],
                a.m[1][1] + b.m[1][1]);
}

// 2D rotation by `rot` radians in the column-major layout used by the
// Image-GS projection: columns (cos, -sin) and (sin, cos).
__device__ __forceinline__ Mat2 rot2(float rot) {
    const float c = cos(rot);
    const float s = sin(rot);
    Mat2 r = mat2_diag(c);
    r.m[0][1] = -s;
    r.m[1][0] = s;
    return r;
}

// Derivative of rot2 with respect to the angle.
__device__ __forceinline__ Mat2 rot2_grad(float rot) {
    const float c = cos(rot);
    const float s = sin(rot);
    Mat2 r = mat2_diag(-s);
    r.m[0][1] = -c;
    r.m[1][0] = c;
    return r;
}

__device__ __forceinline__ Mat2 scale2(float sx, float sy) {
    Mat2 r = mat2_diag(1.f);
    r.m[0][0] = sx;
    r.m[1][1] = sy;
    return r;
}

}  // namespace hx
