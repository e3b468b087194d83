// Real spherical-harmonic basis (degrees 0..4) and its gradient with respect to
// the (already normalised) direction, in the polynomial form of P.-P. Sloan,
// "Efficient Spherical Harmonic Evaluation", JCGT 2013. The numeric constants
// are the standard real-SH normalisation factors, e.g. 1/(2 sqrt(pi)),
// sqrt(3/(4 pi)), (1/2) sqrt(15/pi), ... . Basis ordering and signs match the
// reference (gsplat/cuda/csrc/SphericalHarmonicsCUDA.cu:38-128).
#pragma once

namespace gsb {

constexpr float kSH0 = 0.28209479177387814f;  // 1/(2 sqrt(pi))
constexpr float kSH1 = 0.4886025119029199f;   // sqrt(3/(4 pi))
constexpr float kSH2a = 1.0925484305920792f;  // (1/2) sqrt(15/pi)
constexpr float kSH2b = 0.31539156525252005f; // (1/4) sqrt(5/pi)
constexpr float kSH2c = 0.5462742152960396f;  // (1/4) sqrt(15/pi)
constexpr float kSH3a = 0.5900435899266435f;  // (1/4) sqrt(35/(2 pi))
constexpr float kSH3b = 2.890611442640554f;   // (1/2) sqrt(105/pi)
constexpr float kSH3c = 0.4570457994644658f;  // (1/4) sqrt(21/(2 pi))
constexpr float kSH3d = 0.3731763325901154f;  // (1/4) sqrt(7/pi)
constexpr float kSH3e = 1.445305721320277f;   // (1/4) sqrt(105/pi)
constexpr float kSH4a = 2.5033429417967046f;  // (3/4) sqrt(35/pi)
constexpr float kSH4b = 1.7701307697799304f;  // (3/4) sqrt(35/(2 pi))
constexpr float kSH4c = 0.9461746957575601f;  // (3/4) sqrt(5/pi)
constexpr float kSH4d = 0.6690465435572892f;  // (3/4) sqrt(5/(2 pi))
constexpr float kSH4e = 0.10578554691520431f; // (3/16) sqrt(1/pi)
constexpr float kSH4f = 0.47308734787878f;    // (3/8) sqrt(5/pi)
constexpr float kSH4g = 0.6258357354491761f;  // (3/16) sqrt(35/pi)

// Basis values Y[0 .. (D+1)^2) at unit direction (x, y, z).
template <int D> __device__ __forceinline__ void sh_eval(float x, float y, float z, float *Y) {
    Y[0] = kSH0;
    if (D < 1) return;
    Y[1] = -kSH1 * y;
    Y[2] = kSH1 * z;
    Y[3] = -kSH1 * x;
    if (D < 2) return;
    const float xx = x * x, yy = y * y, zz = z * z;
    const float xy = x * y, yz = y * z, xz = x * z;
    Y[4] = kSH2a * xy;
    Y[5] = -kSH2a * yz;
    Y[6] = kSH2b * (3.f * zz - 1.f);
    Y[7] = -kSH2a * xz;
    Y[8] = kSH2c * (xx - yy);
    if (D < 3) return;
    Y[9] = -kSH3a * y * (3.f * xx - yy);
    Y[10] = kSH3b * xy * z;
    Y[11] = -kSH3c * y * (5.f * zz - 1.f);
    Y[12] = kSH3d * z * (5.f * zz - 3.f);
    Y[13] = -kSH3c * x * (5.f * zz - 1.f);
    Y[14] = kSH3e * z * (xx - yy);
    Y[15] = -kSH3a * x * (xx - 3.f * yy);
    if (D < 4) return;
    Y[16] = kSH4a * xy * (xx - yy);
    Y[17] = -kSH4b * yz * (3.f * xx - yy);
    Y[18] = kSH4c * xy * (7.f * zz - 1.f);
    Y[19] = -kSH4d * yz * (7.f * zz - 3.f);
    Y[20] = kSH4e * (35.f * zz * zz - 30.f * zz + 3.f);
    Y[21] = -kSH4d * xz * (7.f * zz - 3.f);
    Y[22] = kSH4f * (xx - yy) * (7.f * zz - 1.f);
    Y[23] = -kSH4b * xz * (xx - 3.f * yy);
    Y[24] = kSH4g * (xx * xx - 6.f * xx * yy + yy * yy);
}

// Accumulates sum_k w[k] * grad(Y_k) at unit direction (x, y, z) into g[3].
template <int D>
__device__ __forceinline__ void sh_grad_dot(float x, float y, float z, const float *w, float g[3]) {
    g[0] = 0.f;
    g[1] = 0.f;
    g[2] = 0.f;
    if (D < 1) return;
    g[0] += -kSH1 * w[3];
    g[1] += -kSH1 * w[1];
    g[2] += kSH1 * w[2];
    if (D < 2) return;
    const float xx = x * x, yy = y * y, zz = z * z;
    g[0] += kSH2a * (y * w[4] - z * w[7]) + 2.f * kSH2c * x * w[8];
    g[1] += kSH2a * (x * w[4] - z * w[5]) - 2.f * kSH2c * y * w[8];
    g[2] += -kSH2a * (y * w[5] + x * w[7]) + 6.f * kSH2b * z * w[6];
    if (D < 3) return;
    const float d9x = -6.f * kSH3a * x * y, d9y = -3.f * kSH3a * (xx - yy);
    const float d15x = -3.f * kSH3a * (xx - yy), d15y = 6.f * kSH3a * x * y;
    g[0] += d9x * w[9] + kSH3b * y * z * w[10] - kSH3c * (5.f * zz - 1.f) * w[13] +
            2.f * kSH3e * x * z * w[14] + d15x * w[15];
    g[1] += d9y * w[9] + kSH3b * x * z * w[10] - kSH3c * (5.f * zz - 1.f) * w[11] -
            2.f * kSH3e * y * z * w[14] + d15y * w[15];
    g[2] += kSH3b * x * y * w[10] - 10.f * kSH3c * y * z * w[11] +
            kSH3d * (15.f * zz - 3.f) * w[12] - 10.f * kSH3c * x * z * w[13] +
            kSH3e * (xx - yy) * w[14];
    if (D < 4) return;
    const float a7 = 7.f * zz - 1.f, b7 = 7.f * zz - 3.f;
    g[0] += kSH4a * (3.f * xx * y - yy * y) * w[16] - 6.f * kSH4b * x * y * z * w[17] +
            kSH4c * y * a7 * w[18] - kSH4d * z * b7 * w[21] + 2.f * kSH4f * x * a7 * w[22] -
            3.f * kSH4b * z * (xx - yy) * w[23] + kSH4g * (4.f * xx * x - 12.f * x * yy) * w[24];
    g[1] += kSH4a * (xx * x - 3.f * x * yy) * w[16] - 3.f * kSH4b * z * (xx - yy) * w[17] +
            kSH4c * x * a7 * w[18] - kSH4d * z * b7 * w[19] - 2.f * kSH4f * y * a7 * w[22] +
            6.f * kSH4b * x * y * z * w[23] + kSH4g * (4.f * yy * y - 12.f * xx * y) * w[24];
    g[2] += -kSH4b * (3.f * xx * y - yy * y) * w[17] + 14.f * kSH4c * x * y * z * w[18] -
            kSH4d * y * (21.f * zz - 3.f) * w[19] + kSH4e * (140.f * zz * z - 60.f * z) * w[20] -
            kSH4d * x * (21.f * zz - 3.f) * w[21] + 14.f * kSH4f * z * (xx - yy) * w[22] -
            kSH4b * (xx * x - 3.f * x * yy) * w[23];
}

} // namespace gsb
