// Column-major small matrices and vectors for the 3D surfel projection.
//
// Cmat<C, R>::m[c][r] is column c, row r.  The product of A (K columns, R
// rows) and B (C columns, K rows) is summed over the inner index left to
// right, ((a0*b0 + a1*b1) + a2*b2) + a3*b3, and vector helpers use the same
// left-to-right order.  That is the order of the reference's matrix library,
// so the preprocessing arithmetic (and with it tile bounds and counts)
// reproduces the reference bit for bit under the same compiler flags.  Zero
// entries are kept as real entries, not simplified away, for the same reason.
#pragma once

namespace hx {

template <int C, int R>
struct Cmat {
    float m[C][R];
};

template <int C, int K, int R>
__device__ __forceinline__ Cmat<C, R> mmul(const Cmat<K, R>& a, const Cmat<C, K>& b) {
    Cmat<C, R> out;
#pragma unroll
    for (int c = 0; c < C; ++c) {
#pragma unroll
        for (int r = 0; r < R; ++r) {
            float s = a.m[0][r] * b.m[c][0];
#pragma unroll
            for (int k = 1; k < K; ++k) s = s + a.m[k][r] * b.m[c][k];
            out.m[c][r] = s;
        }
    }
    return out;
}

template <int C, int R>
__device__ __forceinline__ Cmat<R, C> mtranspose(const Cmat<C, R>& a) {
    Cmat<R, C> out;
#pragma unroll
    for (int c = 0; c < C; ++c)
#pragma unroll
        for (int r = 0; r < R; ++r) out.m[r][c] = a.m[c][r];
    return out;
}

// Matrix (C columns, R rows) times column vector of length C.
template <int C, int R>
__device__ __forceinline__ void mvec(const Cmat<C, R>& a, const float (&v)[C], float (&out)[R]) {
#pragma unroll
    for (int r = 0; r < R; ++r) {
        float s = a.m[0][r] * v[0];
#pragma unroll
        for (int c = 1; c < C; ++c) s = s + a.m[c][r] * v[c];
        out[r] = s;
    }
}

// Row vector of length R times matrix (C columns, R rows).
template <int C, int R>
__device__ __forceinline__ void vmat(const float (&v)[R], const Cmat<C, R>& a, float (&out)[C]) {
#pragma unroll
    for (int c = 0; c < C; ++c) {
        float s = v[0] * a.m[c][0];
#pragma unroll
        for (int r = 1; r < R; ++r) s = s + v[r] * a.m[c][r];
        out[c] = s;
    }
}

__device__ __forceinline__ float dot3(float ax, float ay, float az, float bx, float by,
                                      float bz) {
    return ax * bx + ay * by + az * bz;
}

// Rotation matrix of a quaternion packed (w, x, y, z) in (q.x, q.y, q.z, q.w),
// normalised with rsqrt.
__device__ __forceinline__ Cmat<3, 3> quat_to_rotmat_wxyz(const float4 q) {
    const float s = rsqrtf(q.w * q.w + q.x * q.x + q.y * q.y + q.z * q.z);
    const float w = q.x * s;
    const float x = q.y * s;
    const float y = q.z * s;
    const float z = q.w * s;
    Cmat<3, 3> R;
    R.m[0][0] = 1.f - 2.f * (y * y + z * z);
    R.m[0][1] = 2.f * (x * y + w * z);
    R.m[0][2] = 2.f * (x * z - w * y);
    R.m[1][0] = 2.f * (x * y - w * z);
    R.m[1][1] = 1.f - 2.f * (x * x + z * z);
    R.m[1][2] = 2.f * (y * z + w * x);
    R.m[2][0] = 2.f * (x * z + w * y);
    R.m[2][1] = 2.f * (y * z - w * x);
    R.m[2][2] = 1.f - 2.f * (x * x + y * y);
    return R;
}

}  // namespace hx
