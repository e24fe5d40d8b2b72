// Per-Gaussian arithmetic of the backward-and-update path.
//
// This translation unit is compiled with -fmad=false: every float/double
// operation below is rounded on its own, in the order written. The CPU oracle
// evaluates the same expressions in the same order, so results agree bit for
// bit (IEEE division and square root on both sides).
//
// Reference semantics followed (file:line in a-elrawy/clad-3dgs):
//   SH basis, degree <= 3, products xy/yz/xz ........ SHGradientConsumer.cu:20-76
//   term VJP wrt direction and coefficients ......... controls/ManualSH.cu:85-112
//   direction -> position VJP ....................... SHGradientConsumer.cu:78-84
//   torch fused-Adam mixed precision ................ SHGradientConsumer.cu:132-143
//   float Adam (AdamConfig) / SGD ................... SHGradientConsumer.cu:92-109
//   quaternion / exp / sigmoid VJPs ................. controls/ManualActivations.cu:20-36,94-100
//   activation Adam .................................. normalization.cu:70-77
#pragma once
#include <cuda_runtime.h>

namespace clad3dgs {

// Real SH normalisation constants (degree 0..3), as used by 3DGS.
constexpr float kC0 = 0.28209479177387814f;
constexpr float kC1 = 0.4886025119029199f;
constexpr float kC2_0 = 1.0925484305920792f;
constexpr float kC2_1 = -1.0925484305920792f;
constexpr float kC2_2 = 0.31539156525252005f;
constexpr float kC2_3 = -1.0925484305920792f;
constexpr float kC2_4 = 0.5462742152960396f;
constexpr float kC3_0 = -0.5900435899266435f;
constexpr float kC3_1 = 2.890611442640554f;
constexpr float kC3_2 = -0.4570457994644658f;
constexpr float kC3_3 = 0.3731763325901154f;
constexpr float kC3_4 = -0.4570457994644658f;
constexpr float kC3_5 = 1.445305721320277f;
constexpr float kC3_6 = -0.5900435899266435f;

// Scaled constants of the basis gradients, rounded once from double.
constexpr float kG9x = (float)(6.0 * (double)kC3_0);
constexpr float kG9y = (float)(3.0 * (double)kC3_0);
constexpr float kG11x = -2.0f * kC3_2;
constexpr float kG11z = 8.0f * kC3_2;
constexpr float kG12xy = (float)(-6.0 * (double)kC3_3);
constexpr float kG13y = -2.0f * kC3_4;
constexpr float kG13z = 8.0f * kC3_4;
constexpr float kG14 = 2.0f * kC3_5;
constexpr float kG15x = (float)(3.0 * (double)kC3_6);
constexpr float kG15y = (float)(-6.0 * (double)kC3_6);

// Direction cosines of one Gaussian seen from the camera, with the shared
// products of the basis.
struct Direction {
  float x, y, z, r;
  float xx, yy, zz, xy, yz, xz;
};

__device__ __forceinline__ Direction make_direction(float px, float py,
                                                    float pz, float cx,
                                                    float cy, float cz) {
  Direction d;
  const float ux = px - cx, uy = py - cy, uz = pz - cz;
  d.r = sqrtf((ux * ux + uy * uy) + uz * uz);
  d.x = ux / d.r;
  d.y = uy / d.r;
  d.z = uz / d.r;
  d.xx = d.x * d.x;
  d.yy = d.y * d.y;
  d.zz = d.z * d.z;
  d.xy = d.x * d.y;
  d.yz = d.y * d.z;
  d.xz = d.x * d.z;
  return d;
}

// Basis value b_J(dir) and its gradient wrt (x, y, z), for a compile-time term.
template <int J>
__device__ __forceinline__ void sh_basis(const Direction& d, float& b,
                                         float& gx, float& gy, float& gz) {
  gx = 0.f;
  gy = 0.f;
  gz = 0.f;
  if constexpr (J == 0) {
    b = kC0;
  } else if constexpr (J == 1) {
    b = -kC1 * d.y;
    gy = -kC1;
  } else if constexpr (J == 2) {
    b = kC1 * d.z;
    gz = kC1;
  } else if constexpr (J == 3) {
    b = -kC1 * d.x;
    gx = -kC1;
  } else if constexpr (J == 4) {
    b = kC2_0 * d.xy;
    gx = kC2_0 * d.y;
    gy = kC2_0 * d.x;
  } else if constexpr (J == 5) {
    b = kC2_1 * d.yz;
    gy = kC2_1 * d.z;
    gz = kC2_1 * d.y;
  } else if constexpr (J == 6) {
    b = kC2_2 * ((2.f * d.zz - d.xx) - d.yy);
    gx = (-2.f * kC2_2) * d.x;
    gy = (-2.f * kC2_2) * d.y;
    gz = (4.f * kC2_2) * d.z;
  } else if constexpr (J == 7) {
    b = kC2_3 * d.xz;
    gx = kC2_3 * d.z;
    gz = kC2_3 * d.x;
  } else if constexpr (J == 8) {
    b = kC2_4 * (d.xx - d.yy);
    gx = (2.f * kC2_4) * d.x;
    gy = (-2.f * kC2_4) * d.y;
  } else if constexpr (J == 9) {
    b = (kC3_0 * d.y) * (3.f * d.xx - d.yy);
    gx = kG9x * d.xy;
    gy = kG9y * (d.xx - d.yy);
  } else if constexpr (J == 10) {
    b = (kC3_1 * d.xy) * d.z;
    gx = kC3_1 * d.yz;
    gy = kC3_1 * d.xz;
    gz = kC3_1 * d.xy;
  } else if constexpr (J == 11) {
    b = (kC3_2 * d.y) * ((4.f * d.zz - d.xx) - d.yy);
    gx = kG11x * d.xy;
    gy = kC3_2 * ((4.f * d.zz - d.xx) - 3.f * d.yy);
    gz = kG11z * d.yz;
  } else if constexpr (J == 12) {
    b = (kC3_3 * d.z) * ((2.f * d.zz - 3.f * d.xx) - 3.f * d.yy);
    gx = kG12xy * d.xz;
    gy = kG12xy * d.yz;
    gz = kC3_3 * ((6.f * d.zz - 3.f * d.xx) - 3.f * d.yy);
  } else if constexpr (J == 13) {
    b = (kC3_4 * d.x) * ((4.f * d.zz - d.xx) - d.yy);
    gx = kC3_4 * ((4.f * d.zz - 3.f * d.xx) - d.yy);
    gy = kG13y * d.xy;
    gz = kG13z * d.xz;
  } else if constexpr (J == 14) {
    b = (kC3_5 * d.z) * (d.xx - d.yy);
    gx = kG14 * d.xz;
    gy = (-kG14) * d.yz;
    gz = kC3_5 * (d.xx - d.yy);
  } else {
    static_assert(J == 15, "SH terms are 0..15");
    b = (kC3_6 * d.x) * (d.xx - 3.f * d.yy);
    gx = kG15x * (d.xx - d.yy);
    gy = kG15y * d.xy;
  }
}

// VJP of dir = (p - c) / |p - c| wrt p, for the direction adjoint s.
__device__ __forceinline__ void direction_vjp(const Direction& d, float sx,
                                              float sy, float sz, float& ox,
                                              float& oy, float& oz) {
  const float ds = (d.x * sx + d.y * sy) + d.z * sz;
  ox = (sx - d.x * ds) / d.r;
  oy = (sy - d.y * ds) / d.r;
  oz = (sz - d.z * ds) / d.r;
}

constexpr double kBeta1 = 0.9, kBeta2 = 0.999, kEps = 1e-15;
constexpr double kOneMinusBeta1 = 1.0 - kBeta1;
constexpr double kOneMinusBeta2 = 1.0 - kBeta2;

// torch fused Adam: double beta arithmetic, float moments, float step size
// (rate / bias1 rounded once), double epsilon added to the float ratio
// sqrt(v) / bias2.
//
// The division by the per-group constant bias2 is evaluated as
// (float)(sqrt(v) * inv_bias2) with inv_bias2 = 1/(double)bias2 rounded to
// double on the host. That is the correctly rounded float quotient: the exact
// quotient of two floats is never a float midpoint and lies at least 2^-49
// (relative) from one, while the double product is within 2^-52 of it, so
// rounding to float lands on the same value (division by a constant known in
// advance; Brisebarre, Muller, Raina, IEEE Trans. Computers 53(8), 2004). The
// oracle divides directly; the bit-exact tests compare the two.
//
// Every product and sum of the moment updates is rounded on its own (the _rn
// intrinsics are never contracted into fused multiply-adds), so the results
// do not depend on the translation unit's -fmad setting.
__device__ __forceinline__ void torch_adam(float& p, float& m, float& v,
                                           float g, float step,
                                           double inv_bias2) {
  const double gd = (double)g;
  m = (float)__dadd_rn(__dmul_rn(kBeta1, (double)m), __dmul_rn(kOneMinusBeta1, gd));
  v = (float)__dadd_rn(__dmul_rn(kBeta2, (double)v),
                       __dmul_rn(__dmul_rn(kOneMinusBeta2, gd), gd));
  const float ratio = (float)((double)sqrtf(v) * inv_bias2);
  // fl32(ratio + 1e-15) equals ratio whenever ratio >= 2^-25: half an ulp of
  // such a ratio is at least 2^-49 (about 1.78e-15), more than 1e-15, even after
  // the intermediate rounding to double. Only smaller ratios need the sum.
  const float denom = ratio >= 0x1p-25f ? ratio : (float)((double)ratio + kEps);
  p = p - (step * m) / denom;
}

// Float Adam with inverse bias corrections (the reference's AdamConfig path).
__device__ __forceinline__ void float_adam(float& p, float& m, float& v,
                                           float g, float rate, float inv1,
                                           float inv2) {
  m = 0.9f * m + 0.1f * g;
  v = 0.999f * v + (0.001f * g) * g;
  p = p - (rate * (m * inv1)) / (sqrtf(v * inv2) + 1e-15f);
}

__device__ __forceinline__ void sgd(float& p, float g) { p = p - 1e-3f * g; }

constexpr float kDcRate = 0.0025f, kRestRate = 0.000125f;

// VJP of q / max(|q|, 1e-12) for all four components; the saved forward norm
// picks the clamp branch and is used on both sides of it.
__device__ __forceinline__ void quaternion_vjp(const float q[4],
                                               const float s[4], float norm,
                                               float out[4]) {
  if (norm < 1e-12f) {
#pragma unroll
    for (int k = 0; k < 4; ++k) out[k] = s[k] / 1e-12f;
    return;
  }
  float qn[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) qn[j] = q[j] / norm;
  float dot = 0.f;
#pragma unroll
  for (int j = 0; j < 4; ++j) dot = dot + qn[j] * s[j];
#pragma unroll
  for (int k = 0; k < 4; ++k) out[k] = (s[k] - qn[k] * dot) / norm;
}

}  // namespace clad3dgs
