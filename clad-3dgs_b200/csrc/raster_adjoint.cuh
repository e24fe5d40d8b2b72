// Adjoints of the Gaussian rasterizer, derived in this package's own notation.
//
// Blend (per pixel, back to front). The forward composites the contributors
// k = 1..n of a pixel as C = sum_k c_k alpha_k T_k + T_{n+1} bg with
// T_{k+1} = T_k (1 - alpha_k). For the loss adjoint dL/dC (= dpix) and the
// per-Gaussian scalar g_k = dpix . c_k (+ dinv * invdepth_k), everything
// behind contributor k enters only through the scalar
//     R_k = sum_{i>k} g_i alpha_i T_i + T_{n+1} (dpix . bg),
// and dC/dalpha_k gives
//     dL/dalpha_k = g_k T_k - R_k / (1 - alpha_k),   R_{k-1} = R_k + g_k alpha_k T_k.
// So the walk keeps two scalars per pixel (T recovered by division, R summed),
// not a colour recurrence. alpha = min(0.99, o G), G = exp(p) with the
// quadratic form p = -1/2 d^T Q d, d = mean - pixel, Q the conic; as in the
// renderer, the cap is not differentiated (dalpha/dG = o). With
// u = dL/dp = o G dL/dalpha:
//     dL/dQ (full symmetric matrix) = -1/2 u d d^T,
//     dL/dmean = -u Q d,      dL/do = G dL/dalpha.
// Both are linear in per-pixel sums, so a thread first sums u d and u d d^T
// over its pixels and applies Q and the -1/2 once per Gaussian
// (`finish_moments`).
//
// Geometry (per Gaussian): Q = S2^-1 with S2 = A S3 A^T + 0.3 I, A = J W.
//   dL/dS2 = -Q Gq Q              (inverse),
//   dL/dS3 = A^T Gs A,  dL/dA = 2 Gs A S3   (congruence, Gs, S3 symmetric),
//   antialiasing: r = det(S2 - 0.3 I) / det(S2), dL/dS2 += dL/dr
//     (det S2 adj(S2 - 0.3 I) - det(S2 - 0.3 I) adj S2) / det(S2)^2,
//   S3 = M M^T, M = R diag(s):  dL/dM = 2 G3 M.
// Output conventions fixed by the renderer interface: dL/dconic stores the
// full-matrix entries (a, b, -, c); dL/dcov3D stores the six upper-triangle
// entries with off-diagonals counted for both symmetric positions; dL/dmean2D
// is with respect to NDC (pixel adjoint times W/2, H/2); the x/z, y/z clamp of
// the Jacobian passes no gradient to the clamped coordinate.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include "raster_math.cuh"

namespace clad3dgs {
namespace raster {

// Field slots of a Gaussian's per-warp adjoint vector (16 slots, the first
// ten used). Before `finish_moments` slots 3..7 hold the moments
// sum u dx, sum u dy, sum u dx^2, sum u dx dy, sum u dy^2.
enum Field : int {
  kRed = 0, kGreen = 1, kBlue = 2,
  kMeanX = 3, kMeanY = 4,
  kConicA = 5, kConicB = 6, kConicC = 7,
  kOpacity = 8, kInvDepth = 9,
  kFields = 10
};

// One pixel's state in the back-to-front walk.
struct PixelWalk {
  float T;         // transmittance in front of the current Gaussian
  float R;         // dL/dC . (everything behind it, background included)
  float dpix[3];   // dL/dC of the pixel
  float dinv;      // dL/d(inverse depth) of the pixel
  uint32_t last;   // one past the pixel's last contributor (0: outside the image)
};

__device__ __forceinline__ void walk_begin(PixelWalk& s, int px, int py, int width,
                                           int height, const float* __restrict__ final_t,
                                           const uint32_t* __restrict__ n_contrib,
                                           const float* __restrict__ dpixels,
                                           const float* __restrict__ dinvdepth_pixels,
                                           const float* __restrict__ bg) {
  const bool inside = px < width && py < height;
  const int pix = py * width + px, hw = width * height;
  s.T = 0.f;
  s.last = 0;
  s.dpix[0] = s.dpix[1] = s.dpix[2] = 0.f;
  s.dinv = 0.f;
  if (inside) {
    s.T = final_t[pix];
    s.last = n_contrib[pix];
    s.dpix[0] = dpixels[pix];
    s.dpix[1] = dpixels[hw + pix];
    s.dpix[2] = dpixels[2 * hw + pix];
    if (dinvdepth_pixels) s.dinv = dinvdepth_pixels[pix];
  }
  s.R = s.T * (bg[0] * s.dpix[0] + bg[1] * s.dpix[1] + bg[2] * s.dpix[2]);
}

// Gaussian number `index` of the tile list (back to front), at offset
// d = mean - pixel from this pixel, p its exponent there (gauss_power). Adds
// the pixel's share to f (moment form) and returns whether it contributed.
// The exponential is taken whether or not the pixel is live, so a walk over
// several pixels branches once per pixel.
__device__ __forceinline__ bool walk_step(PixelWalk& s, uint32_t index, float p, float dx,
                                          float dy, float4 co, const float* rgb3,
                                          float invdepth, float f[16]) {
  const float G = __expf(p);
  const float alpha = fminf(kMaxAlpha, co.w * G);
  if (!(index < s.last && p <= 0.f && alpha >= kMinAlpha)) return false;
  const float keep_inv = 1.f / (1.f - alpha);
  s.T *= keep_inv;                       // T_k from T_{k+1}
  const float w = alpha * s.T;           // the Gaussian's blend weight here
  const float g = s.dpix[0] * rgb3[0] + s.dpix[1] * rgb3[1] + s.dpix[2] * rgb3[2] +
                  s.dinv * invdepth;
  const float dalpha = g * s.T - s.R * keep_inv;
  s.R += g * w;
  const float u = co.w * G * dalpha;     // dL/dp
  f[kRed] += w * s.dpix[0];
  f[kGreen] += w * s.dpix[1];
  f[kBlue] += w * s.dpix[2];
  f[kInvDepth] += w * s.dinv;
  f[kOpacity] += G * dalpha;
  const float udx = u * dx, udy = u * dy;
  f[kMeanX] += udx;
  f[kMeanY] += udy;
  f[kConicA] += udx * dx;
  f[kConicB] += udx * dy;
  f[kConicC] += udy * dy;
  return true;
}

// Moments -> adjoints of the mean (NDC) and conic: dL/dmean = -Q (sum u d),
// dL/dQ = -1/2 sum u d d^T. `half_w`, `half_h` = W/2, H/2.
__device__ __forceinline__ void finish_moments(float f[16], float4 co, float half_w,
                                               float half_h) {
  const float ux = f[kMeanX], uy = f[kMeanY];
  f[kMeanX] = -(co.x * ux + co.y * uy) * half_w;
  f[kMeanY] = -(co.y * ux + co.z * uy) * half_h;
  f[kConicA] *= -0.5f;
  f[kConicB] *= -0.5f;
  f[kConicC] *= -0.5f;
}

// ---------------------------------------------------------------------------
// Warp reductions of the adjoint fields before the global atomics.

// The reference's rule (WarpAccumulation.cuh:9-15): are all 32 lanes active
// and on the same key?
__device__ __forceinline__ bool whole_warp_on(uint32_t key) {
  return __match_any_sync(__activemask(), key) == 0xffffffffu;
}

// Sum over the full warp, delivered to lane 0 (shuffle-down tree).
__device__ __forceinline__ float warp_total_lane0(float v) {
#pragma unroll
  for (int offset = 16; offset; offset >>= 1) v += __shfl_down_sync(0xffffffffu, v, offset);
  return v;
}

// Mode 1: whole warp on one key -> one atomic per field from lane 0; any
// other lane pattern -> one atomic per lane and field. `lane` is the lane id.
template <class Dest>
__device__ __forceinline__ void accumulate_by_key(uint32_t key, const float* f, int fields,
                                                  int lane, Dest dest) {
  const bool whole = whole_warp_on(key);
  for (int q = 0; q < fields; ++q) {
    if (whole) {
      const float total = warp_total_lane0(f[q]);
      if (lane == 0) atomicAdd(dest(q), total);
    } else {
      atomicAdd(dest(q), f[q]);
    }
  }
}

// Sums v[0..9] over the converged warp; afterwards lane L holds the total of
// field (L >> 1) & 15 (lanes L and L ^ 1 hold the same value). Each
// butterfly step halves the fields a lane keeps, so 16 shuffles cover all
// ten fields.
__device__ __forceinline__ float transpose_reduce(float v[16], int lane) {
#pragma unroll
  for (int step = 0; step < 4; ++step) {
    const int half = 8 >> step;   // fields kept after this step
    const int mask = 16 >> step;  // lane bit that picks the half
    const bool upper = lane & mask;
#pragma unroll
    for (int k = 0; k < half; ++k) {
      const float send = upper ? v[k] : v[k + half];
      const float keep = upper ? v[k + half] : v[k];
      v[k] = keep + __shfl_xor_sync(0xffffffffu, send, mask);
    }
  }
  return v[0] + __shfl_xor_sync(0xffffffffu, v[0], 1);
}

// Mode 2: the whole warp is converged on one key (lanes without a share add
// zeros); one transposing reduction, then lanes 0, 2, ..., 2(fields-1) each
// issue the atomic of one field.
template <class Dest>
__device__ __forceinline__ void accumulate_converged(float v[16], int fields, int lane,
                                                     Dest dest) {
  const float total = transpose_reduce(v, lane);
  const int q = (lane >> 1) & 15;
  if ((lane & 1) == 0 && q < fields) atomicAdd(dest(q), total);
}

// ---------------------------------------------------------------------------
// Small symmetric-matrix helpers of the geometry adjoint.

struct Sym2 {
  float xx, xy, yy;
};

// X Y X for symmetric 2x2 X, Y (the inverse adjoint needs -Q G Q).
__device__ __forceinline__ Sym2 sandwich2(Sym2 X, Sym2 Y) {
  // Z = Y X, then X Z.
  const float z00 = Y.xx * X.xx + Y.xy * X.xy, z01 = Y.xx * X.xy + Y.xy * X.yy;
  const float z10 = Y.xy * X.xx + Y.yy * X.xy, z11 = Y.xy * X.xy + Y.yy * X.yy;
  return {X.xx * z00 + X.xy * z10, X.xx * z01 + X.xy * z11, X.xy * z01 + X.yy * z11};
}

// Symmetric 3x3 from its upper triangle (00, 01, 02, 11, 12, 22).
__device__ __forceinline__ void full3(const float u[6], float m[9]) {
  m[0] = u[0]; m[1] = u[1]; m[2] = u[2];
  m[3] = u[1]; m[4] = u[3]; m[5] = u[4];
  m[6] = u[2]; m[7] = u[4]; m[8] = u[5];
}

// d(R(q))/dq contracted with dR (row-major 3x3) for the rotation() of
// raster_math.cuh, q = (w, x, y, z). Each partial of R is linear in q:
//   dR/dw = 2[[0,-z,y],[z,0,-x],[-y,x,0]]
//   dR/dx = 2[[0,y,z],[y,-2x,-w],[z,w,-2x]]
//   dR/dy = 2[[-2y,x,w],[x,0,z],[-w,z,-2y]]
//   dR/dz = 2[[-2z,-w,x],[w,-2z,y],[x,y,0]]
__device__ __forceinline__ void rotation_vjp(const float q[4], const float dR[9],
                                             float out[4]) {
  const float w = q[0], x = q[1], y = q[2], z = q[3];
  const float Pw[9] = {0.f, -z, y, z, 0.f, -x, -y, x, 0.f};
  const float Px[9] = {0.f, y, z, y, -2.f * x, -w, z, w, -2.f * x};
  const float Py[9] = {-2.f * y, x, w, x, 0.f, z, -w, z, -2.f * y};
  const float Pz[9] = {-2.f * z, -w, x, w, -2.f * z, y, x, y, 0.f};
  float sw = 0.f, sx = 0.f, sy = 0.f, sz = 0.f;
#pragma unroll
  for (int k = 0; k < 9; ++k) {
    sw += Pw[k] * dR[k];
    sx += Px[k] * dR[k];
    sy += Py[k] * dR[k];
    sz += Pz[k] * dR[k];
  }
  out[0] = 2.f * sw;
  out[1] = 2.f * sx;
  out[2] = 2.f * sy;
  out[3] = 2.f * sz;
}

}  // namespace raster
}  // namespace clad3dgs
