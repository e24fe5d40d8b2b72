// Device math of the Gaussian rasterizer: projection of 3D Gaussians to screen
// ellipses (EWA splatting), front-to-back alpha compositing and their adjoints.
//
// Written from the published 3D Gaussian Splatting algorithm (Kerbl et al.,
// SIGGRAPH 2023) and EWA volume splatting (Zwicker et al., 2001), following the
// conventions of the renderer the reference plugs into (its argument layout is
// in adapter.py:21-47 and check.py:760-781): column-major 4x4 view and
// projection matrices, quaternions (w, x, y, z), covariance stored as its six
// upper-triangle entries, a 0.3 px^2 low-pass added to the screen covariance
// (optionally compensated in the opacity: "antialiasing"), radius 3 sigma of
// the larger eigenvalue, 16x16 pixel tiles, alpha capped at 0.99 and skipped
// below 1/255, compositing stopped once transmittance would fall below 1e-4.
#pragma once
#include <cuda_runtime.h>

namespace clad3dgs {
namespace raster {

constexpr int kTileX = 16, kTileY = 16, kTilePixels = kTileX * kTileY;
constexpr float kLowPass = 0.3f;
constexpr float kMinAlpha = 1.0f / 255.0f;
constexpr float kMaxAlpha = 0.99f;
constexpr float kMinTransmittance = 0.0001f;
constexpr float kNearPlane = 0.2f;

struct Vec3 {
  float x, y, z;
};

// p' = M [p, 1] with a column-major 4x4 (first three rows).
__device__ __forceinline__ Vec3 affine3(const float* m, Vec3 p) {
  return {m[0] * p.x + m[4] * p.y + m[8] * p.z + m[12],
          m[1] * p.x + m[5] * p.y + m[9] * p.z + m[13],
          m[2] * p.x + m[6] * p.y + m[10] * p.z + m[14]};
}

__device__ __forceinline__ float affine_w(const float* m, Vec3 p) {
  return m[3] * p.x + m[7] * p.y + m[11] * p.z + m[15];
}

// Rotation matrix (row-major) of the quaternion q = (w, x, y, z); q is used as
// given (the caller passes the normalised activation).
__device__ __forceinline__ void rotation(const float q[4], float R[9]) {
  const float w = q[0], x = q[1], y = q[2], z = q[3];
  R[0] = 1.f - 2.f * (y * y + z * z);
  R[1] = 2.f * (x * y - w * z);
  R[2] = 2.f * (x * z + w * y);
  R[3] = 2.f * (x * y + w * z);
  R[4] = 1.f - 2.f * (x * x + z * z);
  R[5] = 2.f * (y * z - w * x);
  R[6] = 2.f * (x * z - w * y);
  R[7] = 2.f * (y * z + w * x);
  R[8] = 1.f - 2.f * (x * x + y * y);
}

// Sigma = R diag(s^2) R^T, upper triangle (00, 01, 02, 11, 12, 22).
__device__ __forceinline__ void covariance3d(const float s[3], const float q[4],
                                             float cov[6]) {
  float R[9];
  rotation(q, R);
  // M = R diag(s): column j of R scaled by s_j; Sigma = M M^T.
  float M[9];
#pragma unroll
  for (int i = 0; i < 3; ++i)
#pragma unroll
    for (int j = 0; j < 3; ++j) M[3 * i + j] = R[3 * i + j] * s[j];
  auto dot = [&](int a, int b) {
    return M[3 * a] * M[3 * b] + M[3 * a + 1] * M[3 * b + 1] + M[3 * a + 2] * M[3 * b + 2];
  };
  cov[0] = dot(0, 0);
  cov[1] = dot(0, 1);
  cov[2] = dot(0, 2);
  cov[3] = dot(1, 1);
  cov[4] = dot(1, 2);
  cov[5] = dot(2, 2);
}

// Rows of A = J W (2x3): the screen-space Jacobian J of the perspective
// projection at the camera-space mean t (x/z, y/z clamped to 1.3 tan(fov)
// as the renderer does), times the camera rotation W.
struct Projection2 {
  float A[6];   // row-major 2x3
  float tx, ty, tz;  // camera-space mean with the clamped x/z, y/z
  bool clamp_x, clamp_y;
};

__device__ __forceinline__ Projection2 screen_jacobian(Vec3 t, float fx, float fy,
                                                       float tan_x, float tan_y,
                                                       const float* view) {
  Projection2 P;
  const float lim_x = 1.3f * tan_x, lim_y = 1.3f * tan_y;
  const float rx = t.x / t.z, ry = t.y / t.z;
  P.clamp_x = rx < -lim_x || rx > lim_x;
  P.clamp_y = ry < -lim_y || ry > lim_y;
  P.tx = fminf(lim_x, fmaxf(-lim_x, rx)) * t.z;
  P.ty = fminf(lim_y, fmaxf(-lim_y, ry)) * t.z;
  P.tz = t.z;
  const float iz = 1.f / t.z, iz2 = iz * iz;
  const float J00 = fx * iz, J02 = -fx * P.tx * iz2;
  const float J11 = fy * iz, J12 = -fy * P.ty * iz2;
  // W: camera rotation, row r of W is (view[r], view[4 + r], view[8 + r]).
#pragma unroll
  for (int c = 0; c < 3; ++c) {
    const float w0 = view[4 * c + 0], w1 = view[4 * c + 1], w2 = view[4 * c + 2];
    P.A[c] = J00 * w0 + J02 * w2;
    P.A[3 + c] = J11 * w1 + J12 * w2;
  }
  return P;
}

// Screen covariance entries (a, b, c) = A Sigma A^T (before the low-pass).
__device__ __forceinline__ void covariance2d(const Projection2& P, const float cov[6],
                                             float& a, float& b, float& c) {
  const float S[9] = {cov[0], cov[1], cov[2], cov[1], cov[3], cov[4],
                      cov[2], cov[4], cov[5]};
  float u0[3], u1[3];  // Sigma A0^T, Sigma A1^T
#pragma unroll
  for (int i = 0; i < 3; ++i) {
    u0[i] = S[3 * i] * P.A[0] + S[3 * i + 1] * P.A[1] + S[3 * i + 2] * P.A[2];
    u1[i] = S[3 * i] * P.A[3] + S[3 * i + 1] * P.A[4] + S[3 * i + 2] * P.A[5];
  }
  a = P.A[0] * u0[0] + P.A[1] * u0[1] + P.A[2] * u0[2];
  b = P.A[0] * u1[0] + P.A[1] * u1[1] + P.A[2] * u1[2];
  c = P.A[3] * u1[0] + P.A[4] * u1[1] + P.A[5] * u1[2];
}

// Exponent p = -1/2 d^T Q d of a Gaussian at offset d = (dx, dy) = mean -
// pixel, Q = [[co.x, co.y], [co.y, co.z]], as a quadratic in dy whose
// coefficients depend only on the pixel column:
//     p = c2 dy^2 + c1 dy + c0,  c2 = -co.z / 2, c1 = -co.y dx, c0 = -co.x dx^2 / 2,
// evaluated by Horner's rule. A thread that shades several rows of one column
// forms (c0, c1, c2) once per Gaussian and spends two fused multiply-adds per
// pixel. Every rounding is explicit, so the forward compositing and the
// backward walk (which must replay the forward's contribution decisions
// exactly) get the same bits whatever the compiler contracts elsewhere.
struct ColumnForm {
  float c0, c1, c2;
};

__device__ __forceinline__ ColumnForm column_form(float4 co, float dx) {
  return {__fmul_rn(-0.5f, __fmul_rn(__fmul_rn(co.x, dx), dx)), -__fmul_rn(co.y, dx),
          -0.5f * co.z};
}

__device__ __forceinline__ float row_power(const ColumnForm& f, float dy) {
  return __fmaf_rn(__fmaf_rn(f.c2, dy, f.c1), dy, f.c0);
}

__device__ __forceinline__ float gauss_power(float4 co, float dx, float dy) {
  return row_power(column_form(co, dx), dy);
}

__device__ __forceinline__ float ndc_to_pixel(float v, int size) {
  return ((v + 1.f) * size - 1.f) * 0.5f;
}

// Tile rectangle [lo, hi) touched by a disc of `radius` px around p.
__device__ __forceinline__ void tile_rect(float px, float py, int radius, int grid_x,
                                          int grid_y, int& x0, int& y0, int& x1,
                                          int& y1) {
  x0 = min(grid_x, max(0, (int)((px - radius) / kTileX)));
  y0 = min(grid_y, max(0, (int)((py - radius) / kTileY)));
  x1 = min(grid_x, max(0, (int)((px + radius + kTileX - 1) / kTileX)));
  y1 = min(grid_y, max(0, (int)((py + radius + kTileY - 1) / kTileY)));
}

// Exact tile footprint. The renderer skips a (pixel, Gaussian) pair when
// alpha = opacity * exp(-q/2) < 1/255, q = A dx^2 + 2B dx dy + C dy^2 with the
// conic (A, B, C) and d = pixel centre - mean. So a tile whose pixel centres all
// have q > tau = 2 ln(255 opacity) receives nothing from the Gaussian and can be
// left out of its instance list without changing any output. Per tile row, the
// pixel-centre band [16 ty, 16 ty + 15] meets the ellipse q <= tau in one x
// interval (the ellipse is convex); its ends come from the ellipse's extreme
// points clamped into the band. tau and the interval carry a margin far above
// float rounding, and the result never leaves the 3-sigma tile rectangle the
// renderer uses, so the kept set always contains every contributing tile.
struct Footprint {
  float mx, my;     // mean, pixels
  float B, invA;    // conic off-diagonal, 1 / A
  float at, detc;   // A tau, A C - B^2
  float ymax, dyr;  // ellipse half-height; dy of its rightmost point
  bool any;         // false: no pixel can contribute
  bool ellipse;     // false: conic not positive definite, keep whole rows
  int x0, y0, x1, y1;  // tile rectangle of the 3-sigma radius
};

// Row-independent terms, once per Gaussian. Every operation is an explicitly
// rounded intrinsic, so the count taken in one kernel and the instances written
// in another agree bit for bit.
__device__ __forceinline__ Footprint make_footprint(float px, float py, float4 co, int radius,
                                                    int grid_x, int grid_y) {
  Footprint f;
  f.mx = px;
  f.my = py;
  const float A = co.x, C = co.z;
  f.B = co.y;
  const float o255 = __fmul_rn(255.f, co.w);
  float tau = o255 > 0.f ? __fmul_rn(2.f, logf(o255)) : -1.f;
  f.any = tau >= 0.f;
  if (f.any) tau = __fadd_rn(__fmul_rn(tau, 1.001f), 0.01f);
  f.detc = __fsub_rn(__fmul_rn(A, C), __fmul_rn(f.B, f.B));
  f.ellipse = A > 0.f && C > 0.f && f.detc > 0.f;
  f.invA = f.ellipse ? __frcp_rn(A) : 0.f;
  f.at = __fmul_rn(A, tau);
  f.ymax = f.ellipse && f.any ? __fsqrt_rn(__fdiv_rn(f.at, f.detc)) : 0.f;
  // Extreme points of the ellipse in x sit at dy = -/+ B sqrt(tau / (C detc)).
  f.dyr = f.ellipse && f.any
              ? __fmul_rn(-f.B, __fsqrt_rn(__fdiv_rn(tau, __fmul_rn(C, f.detc))))
              : 0.f;
  tile_rect(px, py, radius, grid_x, grid_y, f.x0, f.y0, f.x1, f.y1);
  return f;
}

// Tiles [lo, hi) of tile row ty that the footprint reaches (lo >= hi: none).
__device__ __forceinline__ void row_span(const Footprint& f, int ty, int& lo, int& hi) {
  lo = f.x0;
  hi = f.x1;
  if (!f.ellipse) return;
  if (!f.any) {
    hi = lo;
    return;
  }
  constexpr float kPad = 0.05f;  // pixels
  const float a = fmaxf(__fsub_rn(float(ty * kTileY) - kPad, f.my), -f.ymax);
  const float b = fminf(__fsub_rn(float(ty * kTileY + kTileY - 1) + kPad, f.my), f.ymax);
  if (a > b) {
    hi = lo;
    return;
  }
  const float yr = fminf(fmaxf(f.dyr, a), b), yl = fminf(fmaxf(-f.dyr, a), b);
  const float rr = __fsqrt_rn(fmaxf(0.f, __fsub_rn(f.at, __fmul_rn(__fmul_rn(f.detc, yr), yr))));
  const float rl = __fsqrt_rn(fmaxf(0.f, __fsub_rn(f.at, __fmul_rn(__fmul_rn(f.detc, yl), yl))));
  const float xr = __fmul_rn(__fadd_rn(__fmul_rn(-f.B, yr), rr), f.invA);
  const float xl = __fmul_rn(__fsub_rn(__fmul_rn(-f.B, yl), rl), f.invA);
  const float x_hi = __fadd_rn(__fadd_rn(f.mx, xr), kPad);
  const float x_lo = __fsub_rn(__fadd_rn(f.mx, xl), kPad);
  // Tile tx holds pixel centres [16 tx, 16 tx + 15]; x / 16 is exact as x * 0.0625.
  lo = max(lo, (int)ceilf(__fmul_rn(__fsub_rn(x_lo, float(kTileX - 1)), 0.0625f)));
  hi = min(hi, (int)floorf(__fmul_rn(x_hi, 0.0625f)) + 1);
}

__device__ __forceinline__ uint32_t footprint_tiles(const Footprint& f) {
  uint32_t n = 0;
  for (int ty = f.y0; ty < f.y1; ++ty) {
    int lo, hi;
    row_span(f, ty, lo, hi);
    if (hi > lo) n += uint32_t(hi - lo);
  }
  return n;
}

}  // namespace raster
}  // namespace clad3dgs
