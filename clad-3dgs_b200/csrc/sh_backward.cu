// The SH colour and its backward, each in two forms, in one translation unit
// compiled without multiply-add contraction (every product and sum rounded on
// its own, in source order), so that the forms give the same bits:
//
// * the rasterizer's, per view: the colour pass (sh_colour_kernel) and
//   d colour / d coefficients with the view direction's adjoint of every drawn
//   Gaussian (sh_backward_kernel);
// * the data-parallel exchange's, for the SH and position groups of a share
//   (shard_seed_kernel; shard_colour_kernel), below.
//
// Seed form. Every rank renders its own view. Instead of the 48 SH gradients of every
// Gaussian, a rank publishes the colour seed of its view (dL/dcolour with the
// clamped channels zeroed and a drawn flag: 16 bytes) plus the geometry part
// of its position gradient. The owner of a share evaluates, for each of its
// Gaussians and each view q in rank order, the SH backward of view q's colour
// (sh_colour.cuh, the rasterizer's own arithmetic) and the view direction's
// adjoint, sums them as the per-view gradients would be
// summed, and runs torch-fused Adam on the 48 coefficients and 3 positions,
// storing the parameters into every replica. The other groups (scaling,
// rotation, opacity) go through the chunked update of train_step.cu.
//
// Colour form. The owner keeps the updated coefficients in its own replica
// only and, from the rows still in shared memory, renders every rank's colour
// of its Gaussians for that rank's next camera (the colour pass's arithmetic),
// 12 bytes per Gaussian and rank instead of 192; it keeps which channels the
// clamp cut and masks the next seeds with them, as each rank's clamp flags
// masked its seeds in the seed form.
//
// One warp per 32 Gaussians: the warp stages its coefficient block in shared
// memory (rows of 48 floats + 1, so each lane's row starts in its own bank),
// each lane works through its Gaussian's views and leaves the gradient sums in
// its row in place of the coefficients, and the Adam pass over the block is
// coalesced.
#include <cuda_runtime.h>

#include <cstdint>
#include <string>

#include "clad3dgs_b200.h"
#include "gaussian_math.cuh"
#include "sh_colour.cuh"

namespace clad3dgs {
int fail(int code, const std::string& message);  // gaussian_step.cu
}

namespace clad3dgs {
namespace raster {

// Per view: each lane reads coefficient j of its row before overwriting it
// with dL/dsh_j, and the warp stores the dL/dsh block coalesced. The direction
// adjoint is added into dmeans after the geometry backward's share (dmeans is
// zeroed by the caller, so the sum rounds as the single sum would).
__global__ void __launch_bounds__(32 * kShWarps)
    sh_backward_kernel(int P, int degree, const float* __restrict__ means, ShSource sh,
                       const float* __restrict__ campos, const bool* __restrict__ clamped,
                       const int* __restrict__ radii, const float* __restrict__ dcolor,
                       float* __restrict__ dsh, float* __restrict__ dmeans) {
  __shared__ float rows[kShWarps][32 * kShRow];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  float* blk = rows[warp];
  const int i0 = (blockIdx.x * kShWarps + warp) * 32;
  if (i0 >= P) return;  // whole warp
  const int n = min(32, P - i0);
  stage_coefficients(sh, i0, n, lane, blk);
  __syncwarp();
  float* row = blk + lane * kShRow;
  const int i = i0 + lane;
  if (lane < n) {
    if (radii[i] > 0) {
      const Direction d = make_direction(means[3 * i], means[3 * i + 1], means[3 * i + 2],
                                         campos[0], campos[1], campos[2]);
      float gcol[3];
#pragma unroll
      for (int k = 0; k < 3; ++k) gcol[k] = clamped[3 * i + k] ? 0.f : dcolor[3 * i + k];
      float dd[3] = {0.f, 0.f, 0.f};
      colour_adjoint_terms<0>(d, RowSource{row}, i, (degree + 1) * (degree + 1), gcol,
                              CoefficientStore{row}, dd);
      float om[3];
      direction_vjp(d, dd[0], dd[1], dd[2], om[0], om[1], om[2]);
#pragma unroll
      for (int k = 0; k < 3; ++k) dmeans[3 * i + k] = dmeans[3 * i + k] + om[k];
    } else {
#pragma unroll
      for (int k = 0; k < 48; ++k) row[k] = 0.f;
    }
  }
  __syncwarp();
  if (!dsh) return;  // direction adjoint only
  float* dst = dsh + 48 * size_t(i0);
  for (int e = lane; e < n * 48; e += 32) dst[e] = blk[(e / 48) * kShRow + e % 48];
}

// SH colour of every drawn Gaussian (radius > 0): colour + 0.5, clamped at 0,
// with the clamp flags the backward reads (the rasterizer's colour pass).
__global__ void __launch_bounds__(32 * kShWarps)
    sh_colour_kernel(int P, int degree, const float* __restrict__ means, ShSource sh,
                     const float* __restrict__ campos, const int* __restrict__ radii,
                     bool* __restrict__ clamped, float* __restrict__ rgb) {
  __shared__ float rows[kShWarps][32 * kShRow];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  float* blk = rows[warp];
  const int i0 = (blockIdx.x * kShWarps + warp) * 32;
  if (i0 >= P) return;  // whole warp
  const int n = min(32, P - i0);
  stage_coefficients(sh, i0, n, lane, blk);
  __syncwarp();
  const int i = i0 + lane;
  if (lane >= n || radii[i] <= 0) return;
  const Direction d = make_direction(means[3 * i], means[3 * i + 1], means[3 * i + 2],
                                     campos[0], campos[1], campos[2]);
  float c[3];
  bool cut[3];
  shaded_colour(d, RowSource{blk + lane * kShRow}, i, (degree + 1) * (degree + 1), c, cut);
#pragma unroll
  for (int k = 0; k < 3; ++k) {
    clamped[3 * i + k] = cut[k];
    rgb[3 * i + k] = c[k];
  }
}

cudaError_t launch_sh_colour(int P, int degree, const float* means, ShSource sh,
                             const float* campos, const int* radii, bool* clamped, float* rgb,
                             cudaStream_t stream) {
  const int warps = (P + 31) / 32;
  sh_colour_kernel<<<(warps + kShWarps - 1) / kShWarps, 32 * kShWarps, 0, stream>>>(
      P, degree, means, sh, campos, radii, clamped, rgb);
  return cudaGetLastError();
}

cudaError_t launch_sh_backward(int P, int degree, const float* means, ShSource sh,
                               const float* campos, const bool* clamped, const int* radii,
                               const float* dcolor, float* dsh, float* dmeans,
                               cudaStream_t stream) {
  const int warps = (P + 31) / 32;
  sh_backward_kernel<<<(warps + kShWarps - 1) / kShWarps, 32 * kShWarps, 0, stream>>>(
      P, degree, means, sh, campos, clamped, radii, dcolor, dsh, dmeans);
  return cudaGetLastError();
}

}  // namespace raster

namespace train {

constexpr int kSeedWarps = 2;  // 6.3 KB of shared memory per warp
constexpr int kSeedRow = raster::kShRow;
constexpr int kSeedRanks = CLAD3DGS_MAX_RANKS;

struct SeedParams {
  int64_t begin, end;
  int local, nterms;
  const float4* seeds[kSeedRanks];
  const float* cameras[kSeedRanks];
  const float* geo_xyz[kSeedRanks];  // geometry part of each view's position gradient
  float* sh[kSeedRanks];             // parameter replicas [N][48]
  float* xyz[kSeedRanks];            // parameter replicas [N][3]
  float* sh_first;                   // moments of the share
  float* sh_second;
  float* xyz_first;
  float* xyz_second;
  float step_xyz, step_dc, step_rest;
  double inv_bias2;
  // Colour form: the owner renders each rank's next colours [N][3] from its
  // next camera and keeps the clamped channels (bit 3q + k) of its share.
  float* colours[kSeedRanks];
  const float* next_cameras[kSeedRanks];
  uint32_t* clamp_bits;
};

// Several views, term-outer: for each term J every view's contribution to
// d colour / d c_J is formed (views in rank order) and their sum overwrites c_J
// once all views have read it; each view's direction adjoint accumulates in
// dd[q] over the terms in order. The sums and the adjoints are those of the
// view-outer form (one view's SH backward after another), bit for bit.
__device__ __forceinline__ Direction direction_from(float4 u) {
  Direction d;
  d.x = u.x;
  d.y = u.y;
  d.z = u.z;
  d.r = u.w;
  d.xx = d.x * d.x;
  d.yy = d.y * d.y;
  d.zz = d.z * d.z;
  d.xy = d.x * d.y;
  d.yz = d.y * d.z;
  d.xz = d.x * d.z;
  return d;
}

template <int J, int R>
__device__ __forceinline__ void views_adjoint_terms(const float4 (&dir)[R],
                                                    const float3 (&seed)[R], uint32_t drawn,
                                                    float* row, int nterms,
                                                    float (&dd)[R][3]) {
  if constexpr (J < 16) {
    float acc[3];
#pragma unroll
    for (int q = 0; q < R; ++q) {
      float prod[3] = {0.f, 0.f, 0.f};
      if ((drawn >> q & 1u) && J < nterms) {
        float b, gx, gy, gz;
        sh_basis<J>(direction_from(dir[q]), b, gx, gy, gz);
        const float* c = row + 3 * J;
        const float dot = c[0] * seed[q].x + c[1] * seed[q].y + c[2] * seed[q].z;
        dd[q][0] += gx * dot;
        dd[q][1] += gy * dot;
        dd[q][2] += gz * dot;
        prod[0] = b * seed[q].x;
        prod[1] = b * seed[q].y;
        prod[2] = b * seed[q].z;
      }
#pragma unroll
      for (int k = 0; k < 3; ++k) acc[k] = q == 0 ? prod[k] : acc[k] + prod[k];
    }
#pragma unroll
    for (int k = 0; k < 3; ++k) row[3 * J + k] = acc[k];
    views_adjoint_terms<J + 1, R>(dir, seed, drawn, row, nterms, dd);
  }
}

// The block's coefficients into rows of kSeedRow floats, as float4 chunks (a
// chunk never straddles two Gaussians: 48 = 12 x 4), every load independent.
__device__ __forceinline__ void stage_block(const float4* src, int chunks, int lane,
                                            float* cb) {
  for (int c = lane; c < chunks; c += 32) {
    const float4 v = src[c];
    float* dst = cb + (c / 12) * kSeedRow + 4 * (c % 12);
    dst[0] = v.x;
    dst[1] = v.y;
    dst[2] = v.z;
    dst[3] = v.w;
  }
}

// Colour form: Gaussian i's colour from every rank's next camera, by the
// rasterizer's colour pass arithmetic (direction from the position to the
// camera, SH sum + 0.5 clamped at 0; same translation unit, same flags), into
// that rank's colour array, and the clamped channels into the share's bits.
template <int R>
__device__ __forceinline__ void emit_colours(const SeedParams& a, const float (*next)[3],
                                             const float* row, int64_t i,
                                             const float (&pos)[3]) {
  uint32_t bits = 0;
#pragma unroll
  for (int q = 0; q < R; ++q) {
    const Direction d =
        make_direction(pos[0], pos[1], pos[2], next[q][0], next[q][1], next[q][2]);
    float c[3];
    bool cut[3];
    raster::shaded_colour(d, raster::RowSource{row}, int(i), a.nterms, c, cut);
#pragma unroll
    for (int k = 0; k < 3; ++k) {
      __stcs(a.colours[q] + 3 * i + k, c[k]);
      bits |= cut[k] ? 1u << (3 * q + k) : 0u;
    }
  }
  a.clamp_bits[i - a.begin] = bits;
}

// The gradient row overwrites the coefficient row in place (each term's
// coefficients are read, by every view, before its gradients are written) and
// the Adam pass reloads the parameters: one row of shared memory per Gaussian.
// In colour form the Adam pass leaves the new coefficients in the row for the
// next colours, and the coefficients are stored into the owner's replica only.
template <int R, bool Colours>
__global__ void __launch_bounds__(32 * kSeedWarps)
    shard_seed_kernel(const __grid_constant__ SeedParams a) {
  constexpr bool kInPlace = true;
  __shared__ float rows[kSeedWarps][(kInPlace ? 1 : 2) * 32 * kSeedRow];
  __shared__ float cams[R][3];
  __shared__ float next[Colours ? R : 1][3];
  using raster::CoefficientSum;
  using raster::RowSource;
  if (threadIdx.x < 3 * R) {
    const int q = threadIdx.x / 3, k = threadIdx.x % 3;
    cams[q][k] = a.cameras[q][k];
    if (Colours) next[q][k] = a.next_cameras[q][k];
  }
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t i0 = a.begin + (int64_t(blockIdx.x) * kSeedWarps + warp) * 32;
  if (i0 >= a.end) return;  // whole warp
  const int n = int(a.end - i0 < 32 ? a.end - i0 : 32);
  float* cb = rows[warp];
  float* sb = kInPlace ? cb : cb + 32 * kSeedRow;
  const int chunks = n * 12;
  const float4* src = reinterpret_cast<const float4*>(a.sh[a.local] + 48 * i0);
  stage_block(src, chunks, lane, cb);
  // With one or two views the Adam pass's first chunk (moments and
  // parameters) and the position moments are loaded now, so their latency
  // overlaps the SH backward (with more views the registers they hold cost
  // more occupancy than the overlap gains).
  constexpr bool kEarly = R <= 2;
  float4* first = reinterpret_cast<float4*>(a.sh_first + 48 * (i0 - a.begin));
  float4* second = reinterpret_cast<float4*>(a.sh_second + 48 * (i0 - a.begin));
  float4 m4 = make_float4(0.f, 0.f, 0.f, 0.f), v4 = m4, p4 = m4;
  if (kEarly && lane < chunks) {
    m4 = first[lane];
    v4 = second[lane];
    if (kInPlace) p4 = src[lane];
  }
  __syncwarp();
  float moved[3] = {0.f, 0.f, 0.f};  // the updated position (colour form)
  if (lane < n) {
    const int64_t i = i0 + lane;
    const float* row = cb + lane * kSeedRow;
    float* sum = sb + lane * kSeedRow;
    float pos[3], xm[3] = {0.f, 0.f, 0.f}, xv[3] = {0.f, 0.f, 0.f};
    const int64_t mx = 3 * (i - a.begin);
#pragma unroll
    for (int k = 0; k < 3; ++k) {
      pos[k] = a.xyz[a.local][3 * i + k];
      if (kEarly) {
        xm[k] = a.xyz_first[mx + k];
        xv[k] = a.xyz_second[mx + k];
      }
    }
    // Every view's seed first (independent loads, many in flight over
    // NVLink); with one view its geometry gradient too (with several, those
    // loads wait until the SH backward is done: fewer live registers).
    float4 seed[R];
    float geo[1][3];
#pragma unroll
    for (int q = 0; q < R; ++q) seed[q] = a.seeds[q][i];
    if constexpr (R == 1) {
#pragma unroll
      for (int k = 0; k < 3; ++k) geo[0][k] = a.geo_xyz[0][3 * i + k];
    }
    if constexpr (Colours) {
      // View q rendered the colours this owner made for it: its seed carries
      // every channel, and the channels the clamp cut have no gradient.
      const uint32_t bits = a.clamp_bits[i - a.begin];
#pragma unroll
      for (int q = 0; q < R; ++q) {
        if (bits & (1u << (3 * q))) seed[q].x = 0.f;
        if (bits & (1u << (3 * q + 1))) seed[q].y = 0.f;
        if (bits & (1u << (3 * q + 2))) seed[q].z = 0.f;
      }
    }
    float x[3];
    if constexpr (R > 1) {
      float4 dir[R];
      float3 colour_seed[R];
      float dd[R][3];
      uint32_t drawn = 0;
#pragma unroll
      for (int q = 0; q < R; ++q) {
        dir[q] = make_float4(0.f, 0.f, 0.f, 1.f);
        colour_seed[q] = make_float3(seed[q].x, seed[q].y, seed[q].z);
        if (seed[q].w != 0.f) {
          drawn |= 1u << q;
          const Direction d = make_direction(pos[0], pos[1], pos[2], cams[q][0], cams[q][1],
                                             cams[q][2]);
          dir[q] = make_float4(d.x, d.y, d.z, d.r);
        }
        dd[q][0] = dd[q][1] = dd[q][2] = 0.f;
      }
      views_adjoint_terms<0, R>(dir, colour_seed, drawn, sum, a.nterms, dd);
      float geo_q[R][3];
#pragma unroll
      for (int q = 0; q < R; ++q)
#pragma unroll
        for (int k = 0; k < 3; ++k) geo_q[q][k] = a.geo_xyz[q][3 * i + k];
#pragma unroll
      for (int q = 0; q < R; ++q) {
        float xq[3] = {geo_q[q][0], geo_q[q][1], geo_q[q][2]};
        if (drawn >> q & 1u) {
          float om[3];
          direction_vjp(direction_from(dir[q]), dd[q][0], dd[q][1], dd[q][2], om[0], om[1],
                        om[2]);
#pragma unroll
          for (int k = 0; k < 3; ++k) xq[k] = geo_q[q][k] + om[k];
        }
#pragma unroll
        for (int k = 0; k < 3; ++k) x[k] = q == 0 ? xq[k] : x[k] + xq[k];
      }
    } else {
#pragma unroll
    for (int q = 0; q < R; ++q) {
      float xq[3];
      if (seed[q].w != 0.f) {
        const Direction d = make_direction(pos[0], pos[1], pos[2], cams[q][0], cams[q][1],
                                           cams[q][2]);
        const float g3[3] = {seed[q].x, seed[q].y, seed[q].z};
        float dd[3] = {0.f, 0.f, 0.f};
        raster::colour_adjoint_terms<0>(d, RowSource{row}, int(i), a.nterms, g3,
                                        CoefficientSum{sum, q == 0}, dd);
        float om[3];
        direction_vjp(d, dd[0], dd[1], dd[2], om[0], om[1], om[2]);
#pragma unroll
        for (int k = 0; k < 3; ++k) xq[k] = geo[q][k] + om[k];
      } else {
        // Not drawn in view q: its SH gradient is zero and its position
        // gradient the geometry part alone.
        for (int k = 0; k < 48; ++k) sum[k] = q == 0 ? 0.f : sum[k] + 0.f;
#pragma unroll
        for (int k = 0; k < 3; ++k) xq[k] = geo[q][k];
      }
#pragma unroll
      for (int k = 0; k < 3; ++k) x[k] = q == 0 ? xq[k] : x[k] + xq[k];
    }
    }
#pragma unroll
    for (int k = 0; k < 3; ++k) {
      float p = pos[k], m = kEarly ? xm[k] : a.xyz_first[mx + k];
      float v = kEarly ? xv[k] : a.xyz_second[mx + k];
      torch_adam(p, m, v, x[k], a.step_xyz, a.inv_bias2);
      a.xyz_first[mx + k] = m;
      a.xyz_second[mx + k] = v;
      moved[k] = p;
#pragma unroll
      for (int q = 0; q < R; ++q) __stcs(a.xyz[q] + 3 * i + k, p);
    }
  }
  __syncwarp();
  // Adam over the block's coefficients in float4 chunks, coalesced; each
  // lane loads its next chunk's moments before updating the current one.
  if (!kEarly && lane < chunks) {
    m4 = first[lane];
    v4 = second[lane];
    if (kInPlace) p4 = src[lane];
  }
  for (int c = lane; c < chunks; c += 32) {
    float4 m_next = m4, v_next = v4, p_next = p4;
    if (c + 32 < chunks) {
      m_next = first[c + 32];
      v_next = second[c + 32];
      if (kInPlace) p_next = src[c + 32];
    }
    const int j = 4 * (c % 12), at = (c / 12) * kSeedRow + j;
    float p[4];
    if (kInPlace) {
      p[0] = p4.x, p[1] = p4.y, p[2] = p4.z, p[3] = p4.w;
    } else {
      p[0] = cb[at], p[1] = cb[at + 1], p[2] = cb[at + 2], p[3] = cb[at + 3];
    }
    float m[4] = {m4.x, m4.y, m4.z, m4.w}, v[4] = {v4.x, v4.y, v4.z, v4.w};
#pragma unroll
    for (int t = 0; t < 4; ++t)
      torch_adam(p[t], m[t], v[t], sb[at + t], j + t < 3 ? a.step_dc : a.step_rest,
                 a.inv_bias2);
    first[c] = make_float4(m[0], m[1], m[2], m[3]);
    second[c] = make_float4(v[0], v[1], v[2], v[3]);
    const float4 out = make_float4(p[0], p[1], p[2], p[3]);
    if constexpr (Colours) {
      // This lane alone read these gradient elements: the row takes the new
      // coefficients in their place.
#pragma unroll
      for (int t = 0; t < 4; ++t) sb[at + t] = p[t];
      __stcs(reinterpret_cast<float4*>(a.sh[a.local] + 48 * i0) + c, out);
    } else {
#pragma unroll
      for (int q = 0; q < R; ++q)
        __stcs(reinterpret_cast<float4*>(a.sh[q] + 48 * i0) + c, out);
    }
    m4 = m_next;
    v4 = v_next;
    p4 = p_next;
  }
  if constexpr (Colours) {
    __syncwarp();
    if (lane < n) emit_colours<R>(a, next, sb + lane * kSeedRow, i0 + lane, moved);
  }
  // Make the peer stores visible system-wide before the kernel retires.
  if (R > 1) __threadfence_system();
}

// Colour form, before the first update: the share's colours from the current
// positions and coefficients of the owner's replica.
template <int R>
__global__ void __launch_bounds__(32 * kSeedWarps)
    shard_colour_kernel(const __grid_constant__ SeedParams a) {
  __shared__ float rows[kSeedWarps][32 * kSeedRow];
  __shared__ float next[R][3];
  if (threadIdx.x < 3 * R) next[threadIdx.x / 3][threadIdx.x % 3] =
      a.next_cameras[threadIdx.x / 3][threadIdx.x % 3];
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t i0 = a.begin + (int64_t(blockIdx.x) * kSeedWarps + warp) * 32;
  if (i0 >= a.end) return;  // whole warp
  const int n = int(a.end - i0 < 32 ? a.end - i0 : 32);
  float* cb = rows[warp];
  stage_block(reinterpret_cast<const float4*>(a.sh[a.local] + 48 * i0), n * 12, lane, cb);
  __syncwarp();
  if (lane < n) {
    const int64_t i = i0 + lane;
    float pos[3];
#pragma unroll
    for (int k = 0; k < 3; ++k) pos[k] = a.xyz[a.local][3 * i + k];
    emit_colours<R>(a, next, cb + lane * kSeedRow, i, pos);
  }
  if (R > 1) __threadfence_system();
}

template <int R>
cudaError_t launch_seed(const SeedParams& p, bool colours, bool update, cudaStream_t stream) {
  const int64_t warps = (p.end - p.begin + 31) / 32;
  const unsigned blocks = unsigned((warps + kSeedWarps - 1) / kSeedWarps);
  if (!update)
    shard_colour_kernel<R><<<blocks, 32 * kSeedWarps, 0, stream>>>(p);
  else if (colours)
    shard_seed_kernel<R, true><<<blocks, 32 * kSeedWarps, 0, stream>>>(p);
  else
    shard_seed_kernel<R, false><<<blocks, 32 * kSeedWarps, 0, stream>>>(p);
  return cudaGetLastError();
}

bool aligned16(const void* p);  // train_step.cu

cudaError_t launch_for(const SeedParams& p, int ranks, bool colours, bool update,
                       cudaStream_t stream) {
  switch (ranks) {
    case 1: return launch_seed<1>(p, colours, update, stream);
    case 2: return launch_seed<2>(p, colours, update, stream);
    case 3: return launch_seed<3>(p, colours, update, stream);
    case 4: return launch_seed<4>(p, colours, update, stream);
    case 5: return launch_seed<5>(p, colours, update, stream);
    case 6: return launch_seed<6>(p, colours, update, stream);
    case 7: return launch_seed<7>(p, colours, update, stream);
    default: return launch_seed<8>(p, colours, update, stream);
  }
}

// The colour form's fields: a colour array and a next camera per rank, the
// share's clamp bits.
int colour_fields(const clad3dgs_shard_update_args& x, SeedParams& p) {
  for (int q = 0; q < x.ranks; ++q) {
    if (!x.colours[q] || !x.next_cameras[q])
      return fail(CLAD3DGS_INVALID_ARGUMENT,
                  "shard update: the colour form needs every rank's colour array and next "
                  "camera");
    p.colours[q] = x.colours[q];
    p.next_cameras[q] = x.next_cameras[q];
  }
  if (!x.clamp_bits)
    return fail(CLAD3DGS_INVALID_ARGUMENT, "shard update: the colour form needs clamp bits");
  p.clamp_bits = x.clamp_bits;
  return CLAD3DGS_OK;
}

// The SH and position groups of clad3dgs_shard_update in seed (or colour)
// form (the arguments are validated by the caller, except the seed fields).
int shard_seed_update(const clad3dgs_shard_update_args& x, cudaStream_t stream) {
  if (x.degree < 0 || x.degree > 3)
    return fail(CLAD3DGS_INVALID_ARGUMENT, "shard update: SH degree must be 0..3");
  if (x.grad_origin != 0)
    return fail(CLAD3DGS_INVALID_ARGUMENT,
                "shard update: the seed form needs full gradient arrays (grad_origin 0)");
  SeedParams p{};
  p.begin = x.begin;
  p.end = x.end;
  p.local = x.local;
  p.nterms = (x.degree + 1) * (x.degree + 1);
  for (int q = 0; q < x.ranks; ++q) {
    if (!x.seeds[q] || !x.cameras[q] || !aligned16(x.seeds[q]))
      return fail(CLAD3DGS_INVALID_ARGUMENT,
                  "shard update: every rank needs a 16-byte aligned seed array and a camera");
    p.seeds[q] = reinterpret_cast<const float4*>(x.seeds[q]);
    p.cameras[q] = x.cameras[q];
    p.geo_xyz[q] = x.grads[q][0];
    p.sh[q] = x.params[q][1];
    p.xyz[q] = x.params[q][0];
  }
  const bool colours = x.colours[0] != nullptr;
  if (colours) {
    const int status = colour_fields(x, p);
    if (status != CLAD3DGS_OK) return status;
  }
  p.sh_first = x.first[1];
  p.sh_second = x.second[1];
  p.xyz_first = x.first[0];
  p.xyz_second = x.second[0];
  p.step_xyz = float(x.rates[0] / double(x.bias1));
  p.step_dc = float(x.rates[1] / double(x.bias1));
  p.step_rest = float(x.rates[2] / double(x.bias1));
  p.inv_bias2 = 1.0 / double(x.bias2_sqrt);
  const cudaError_t e = launch_for(p, x.ranks, colours, true, stream);
  return e == cudaSuccess ? CLAD3DGS_OK
                          : fail(CLAD3DGS_CUDA_ERROR, std::string("shard update (seeds): ") +
                                                          cudaGetErrorString(e));
}

}  // namespace train
}  // namespace clad3dgs

using namespace clad3dgs;
using namespace clad3dgs::train;

extern "C" int clad3dgs_shard_colours(const clad3dgs_shard_update_args* args,
                                      cudaStream_t stream) {
  if (!args) return fail(CLAD3DGS_INVALID_ARGUMENT, "shard colours: null arguments");
  const clad3dgs_shard_update_args& x = *args;
  if (x.ranks < 1 || x.ranks > kSeedRanks)
    return fail(CLAD3DGS_INVALID_ARGUMENT, "shard colours: ranks must be 1..8");
  if (x.local < 0 || x.local >= x.ranks)
    return fail(CLAD3DGS_INVALID_ARGUMENT, "shard colours: local replica out of range");
  if (x.begin < 0 || x.end < x.begin)
    return fail(CLAD3DGS_INVALID_ARGUMENT, "shard colours: range must be ordered");
  if (x.degree < 0 || x.degree > 3)
    return fail(CLAD3DGS_INVALID_ARGUMENT, "shard colours: SH degree must be 0..3");
  if (!x.params[x.local][0] || !x.params[x.local][1] || !aligned16(x.params[x.local][1]))
    return fail(CLAD3DGS_INVALID_ARGUMENT,
                "shard colours: the local positions and 16-byte aligned coefficients are "
                "needed");
  if (x.end == x.begin) return CLAD3DGS_OK;
  SeedParams p{};
  p.begin = x.begin;
  p.end = x.end;
  p.local = x.local;
  p.nterms = (x.degree + 1) * (x.degree + 1);
  p.sh[x.local] = x.params[x.local][1];
  p.xyz[x.local] = x.params[x.local][0];
  const int status = colour_fields(x, p);
  if (status != CLAD3DGS_OK) return status;
  const cudaError_t e = launch_for(p, x.ranks, true, false, stream);
  return e == cudaSuccess ? CLAD3DGS_OK
                          : fail(CLAD3DGS_CUDA_ERROR, std::string("shard colours: ") +
                                                          cudaGetErrorString(e));
}
