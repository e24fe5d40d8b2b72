// View-dependent colour of a Gaussian from its spherical-harmonics
// coefficients (degree <= 3, [16][3] per Gaussian) and the adjoints of that
// colour: d colour / d coefficients and the adjoint of the view direction.
//
// The colour is sum_j basis_j(dir) * c_j over the active terms j < (deg+1)^2
// (the 3DGS convention: the renderer adds 0.5 and clamps at 0 afterwards).
// Used by the rasterizer's colour forward (rasterizer.cu) and by both forms of
// the SH backward, the rasterizer's per view and the data-parallel exchange's
// over every view's colour seed (sh_backward.cu, one translation unit compiled
// without multiply-add contraction, so the two forms round exactly alike).
#pragma once
#include <cuda_runtime.h>

#include <cstddef>

#include "gaussian_math.cuh"

namespace clad3dgs {
namespace raster {

// SH colour access for packed [P][16][3] or split dc [P][3] + rest [P][45].
struct ShSource {
  const float* packed;
  const float* dc;
  const float* rest;
  __device__ __forceinline__ const float* term(int i, int j) const {
    if (packed) return packed + 48 * size_t(i) + 3 * j;
    return j == 0 ? dc + 3 * size_t(i) : rest + 45 * size_t(i) + 3 * (j - 1);
  }
};

// The SH kernels work on 32 Gaussians per warp: the warp stages its block of
// coefficients in shared memory with coalesced loads (rows of 48 floats + 1,
// so rows start in distinct banks) and each lane works in its own row.
constexpr int kShRow = 49;
constexpr int kShWarps = 4;

__device__ __forceinline__ void stage_coefficients(const ShSource& sh, int i0, int n, int lane,
                                                   float* blk) {
  if (sh.packed) {
    const float* src = sh.packed + 48 * size_t(i0);
    for (int e = lane; e < n * 48; e += 32) blk[(e / 48) * kShRow + e % 48] = src[e];
  } else {
    const float* dc = sh.dc + 3 * size_t(i0);
    const float* rest = sh.rest + 45 * size_t(i0);
    for (int e = lane; e < n * 3; e += 32) blk[(e / 3) * kShRow + e % 3] = dc[e];
    for (int e = lane; e < n * 45; e += 32) blk[(e / 45) * kShRow + 3 + e % 45] = rest[e];
  }
}

// Coefficients of one Gaussian staged in a shared-memory row ([16][3]).
struct RowSource {
  const float* row;
  __device__ __forceinline__ const float* term(int, int j) const { return row + 3 * j; }
};

template <int J, class Source>
__device__ __forceinline__ void colour_terms(const Direction& d, const Source& sh, int i,
                                             int nterms, float rgb[3]) {
  if constexpr (J < 16) {
    if (J < nterms) {
      float b, gx, gy, gz;
      sh_basis<J>(d, b, gx, gy, gz);
      const float* c = sh.term(i, J);
      rgb[0] += b * c[0];
      rgb[1] += b * c[1];
      rgb[2] += b * c[2];
      colour_terms<J + 1>(d, sh, i, nterms, rgb);
    }
  }
}

// The rendered colour of one Gaussian seen along d: the SH colour + 0.5,
// clamped at 0, and which channels the clamp cut (their colour adjoint is
// dropped by the backward). The forward's colour pass and the data-parallel
// owner's colour production (sh_backward.cu) both call this from one
// translation unit, so they give the same bits.
template <class Source>
__device__ __forceinline__ void shaded_colour(const Direction& d, const Source& sh, int i,
                                              int nterms, float rgb[3], bool clamped[3]) {
  float sum[3] = {0.f, 0.f, 0.f};
  colour_terms<0>(d, sh, i, nterms, sum);
#pragma unroll
  for (int k = 0; k < 3; ++k) {
    const float v = sum[k] + 0.5f;
    clamped[k] = v < 0.f;
    rgb[k] = fmaxf(v, 0.f);
  }
}

// Where d colour / d c_j goes: stored (null: not wanted), or added to a sum
// over views (`first`: the sum starts here). The sum rounds each product
// before adding it, as a sum of stored per-view adjoints would (and as every
// operation does where contraction is off).
struct CoefficientStore {
  float* dsh;
  __device__ __forceinline__ bool on() const { return dsh != nullptr; }
  __device__ __forceinline__ void put(int k, float v) const { dsh[k] = v; }
};

struct CoefficientSum {
  float* acc;
  bool first;
  __device__ __forceinline__ bool on() const { return true; }
  __device__ __forceinline__ void put(int k, float v) const {
    acc[k] = first ? v : __fadd_rn(acc[k], v);
  }
};

// SH backward for one Gaussian: d colour / d coefficients (into `out`) and the
// adjoint of the view direction (added into dd).
template <int J, class Source, class Out>
__device__ __forceinline__ void colour_adjoint_terms(const Direction& d, const Source& sh,
                                                     int i, int nterms, const float g[3],
                                                     const Out& out, float dd[3]) {
  if constexpr (J < 16) {
    float b, gx, gy, gz;
    sh_basis<J>(d, b, gx, gy, gz);
    if (J < nterms) {
      const float* c = sh.term(i, J);
      const float dot = c[0] * g[0] + c[1] * g[1] + c[2] * g[2];
      dd[0] += gx * dot;
      dd[1] += gy * dot;
      dd[2] += gz * dot;
      if (out.on()) {
        out.put(3 * J, b * g[0]);
        out.put(3 * J + 1, b * g[1]);
        out.put(3 * J + 2, b * g[2]);
      }
    } else if (out.on()) {
      out.put(3 * J, 0.f);
      out.put(3 * J + 1, 0.f);
      out.put(3 * J + 2, 0.f);
    }
    colour_adjoint_terms<J + 1>(d, sh, i, nterms, g, out, dd);
  }
}

}  // namespace raster
}  // namespace clad3dgs
