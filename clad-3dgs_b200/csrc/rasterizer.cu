// Tile-based Gaussian rasterizer for B200: projection, binning, forward
// compositing, and the backward pass whose pixel stage accumulates per-Gaussian
// adjoints with warp reductions before the global atomics.
//
// Pipeline (forward): preprocess (one thread per Gaussian: camera transform,
// 3D covariance from scale and rotation, EWA screen covariance, conic, radius,
// the tiles its alpha >= 1/255 footprint reaches, SH colour and its clamp
// flags) -> depth order -> per-tile lists of Gaussian ids in depth order,
// built from (tile row, depth rank) pairs without sorting per-instance keys
// (see "Binning") -> compositing (one 16x16 CTA per tile, Gaussians staged in
// shared memory in batches of 256).
//
// Pixel backward: the same traversal back to front, starting at the tile's
// largest last-contributor index rather than the end of its range. Every pixel contributes
// ten adjoints per Gaussian (RGB, screen mean x/y, conic a/b/c, opacity,
// inverse depth). Accumulation modes:
//   0  one atomic per contributing lane and adjoint (the unpatched renderer);
//   1  the reference's WarpAccumulation.cuh: a shuffle reduction and one
//      atomic per adjoint when all 32 lanes contribute to the same Gaussian,
//      per-lane atomics otherwise (WarpAccumulation.cuh:9-29);
//   2  (default) all lanes stay converged on each Gaussian, lanes that do not
//      contribute add zeros, and a transposing butterfly (16 shuffles instead
//      of 10 x 5) leaves each of the ten sums in one lane pair, so a warp
//      issues a single 10-lane atomic instruction per Gaussian it touches,
//      partial warps included.
// All three give the same gradients up to floating-point summation order.
//
// Geometry backward (one thread per Gaussian): conic -> screen covariance ->
// 3D covariance (and the mean through the projection Jacobian), covariance ->
// scale and rotation, screen mean and inverse depth -> 3D mean, and SH colour
// -> coefficients and view direction, unless the SH adjoint is consumed by the
// fused SH + Adam kernel instead (see gaussian_step.cu).
#include <cub/cub.cuh>

#include <algorithm>
#include <climits>
#include <cstdint>
#include <string>

#include "clad3dgs_b200.h"
#include "gaussian_math.cuh"
#include "raster_adjoint.cuh"
#include "raster_math.cuh"
#include "sh_colour.cuh"

namespace clad3dgs {
int fail(int code, const std::string& message);  // gaussian_step.cu
}

namespace clad3dgs {
namespace raster {

constexpr int kBatch = kTilePixels;

template <class T>
__host__ __device__ inline size_t aligned(size_t v) {
  return (v + 127) & ~size_t(127);
}

// ---------------------------------------------------------------------------
// Buffer layouts carved out of caller-provided memory.

struct GeomState {
  float* depth;          // camera z
  bool* clamped;         // [P][3]
  int* radii;            // internal copy
  float2* mean2d;        // pixel coordinates
  float* cov3d;          // [P][6]
  float4* conic_opacity; // conic (a, b, c), opacity x antialias factor
  float* rgb;            // [P][3]
  uint32_t* tiles;       // tiles touched (footprint)
  uint32_t* rows;        // rows of the tile rectangle (0 without tiles)
  uint32_t* offsets;     // inclusive scan of rows, in depth order
  uint32_t* totals;      // [2]: tile instances, row pairs
  uint32_t* depth_keys;  // depth bits (then tiles touched in depth order)
  uint32_t* ids;         // 0..P-1
  uint32_t* depth_sorted;
  uint32_t* order;       // Gaussian ids by increasing depth
  void* scan_tmp;
  size_t scan_bytes;
  void* order_tmp;
  size_t order_bytes;
};

size_t scan_temp_bytes(int P) {
  size_t scan = 0, sum = 0;
  cub::DeviceScan::InclusiveSum(nullptr, scan, (uint32_t*)nullptr, (uint32_t*)nullptr, P);
  cub::DeviceReduce::Sum(nullptr, sum, (uint32_t*)nullptr, (uint32_t*)nullptr, P);
  return scan > sum ? scan : sum;
}

size_t order_temp_bytes(int P) {
  size_t bytes = 0;
  cub::DeviceRadixSort::SortPairs(nullptr, bytes, (uint32_t*)nullptr, (uint32_t*)nullptr,
                                  (uint32_t*)nullptr, (uint32_t*)nullptr, P, 0, 32);
  return bytes;
}

size_t geom_bytes(int P) {
  size_t s = 0;
  s += aligned<float>(sizeof(float) * P);
  s += aligned<bool>(3 * P);
  s += aligned<int>(sizeof(int) * P);
  s += aligned<float2>(sizeof(float2) * P);
  s += aligned<float>(sizeof(float) * 6 * P);
  s += aligned<float4>(sizeof(float4) * P);
  s += aligned<float>(sizeof(float) * 3 * P);
  s += 7 * aligned<uint32_t>(sizeof(uint32_t) * P) + aligned<uint32_t>(8);
  s += aligned<char>(scan_temp_bytes(P));
  s += aligned<char>(order_temp_bytes(P));
  return s + 128;
}

GeomState geom_from(char* base, int P) {
  GeomState g;
  char* c = reinterpret_cast<char*>((reinterpret_cast<uintptr_t>(base) + 127) & ~uintptr_t(127));
  auto take = [&](size_t bytes) {
    char* r = c;
    c += aligned<char>(bytes);
    return r;
  };
  g.depth = reinterpret_cast<float*>(take(sizeof(float) * P));
  g.clamped = reinterpret_cast<bool*>(take(3 * P));
  g.radii = reinterpret_cast<int*>(take(sizeof(int) * P));
  g.mean2d = reinterpret_cast<float2*>(take(sizeof(float2) * P));
  g.cov3d = reinterpret_cast<float*>(take(sizeof(float) * 6 * P));
  g.conic_opacity = reinterpret_cast<float4*>(take(sizeof(float4) * P));
  g.rgb = reinterpret_cast<float*>(take(sizeof(float) * 3 * P));
  g.tiles = reinterpret_cast<uint32_t*>(take(sizeof(uint32_t) * P));
  g.rows = reinterpret_cast<uint32_t*>(take(sizeof(uint32_t) * P));
  g.offsets = reinterpret_cast<uint32_t*>(take(sizeof(uint32_t) * P));
  g.totals = reinterpret_cast<uint32_t*>(take(8));
  g.depth_keys = reinterpret_cast<uint32_t*>(take(sizeof(uint32_t) * P));
  g.ids = reinterpret_cast<uint32_t*>(take(sizeof(uint32_t) * P));
  g.depth_sorted = reinterpret_cast<uint32_t*>(take(sizeof(uint32_t) * P));
  g.order = reinterpret_cast<uint32_t*>(take(sizeof(uint32_t) * P));
  g.scan_bytes = scan_temp_bytes(P);
  g.scan_tmp = take(g.scan_bytes);
  g.order_bytes = order_temp_bytes(P);
  g.order_tmp = take(g.order_bytes);
  return g;
}

struct ImageState {
  uint2* ranges;        // per tile
  uint32_t* n_contrib;  // per pixel
  float* final_t;       // per pixel
};

size_t image_bytes(int pixels, int tiles) {
  return aligned<uint2>(sizeof(uint2) * tiles) + aligned<uint32_t>(4 * size_t(pixels)) +
         aligned<float>(4 * size_t(pixels)) + 128;
}

ImageState image_from(char* base, int pixels, int tiles) {
  ImageState s;
  char* c = reinterpret_cast<char*>((reinterpret_cast<uintptr_t>(base) + 127) & ~uintptr_t(127));
  s.ranges = reinterpret_cast<uint2*>(c);
  c += aligned<uint2>(sizeof(uint2) * tiles);
  s.n_contrib = reinterpret_cast<uint32_t*>(c);
  c += aligned<uint32_t>(4 * size_t(pixels));
  s.final_t = reinterpret_cast<float*>(c);
  return s;
}

// Binning buffer: the point list (Gaussian ids grouped by tile, in depth order)
// first, so the backward finds it at the start; then the forward's scratch.
struct BinningState {
  uint32_t* values;          // [n]
  uint32_t* pair_rows;       // [m] row pairs: key tile row, value packed span
  uint32_t* pair_rows_sorted;
  uint64_t* pair_spans;
  uint64_t* pair_spans_sorted;
  void* sort_tmp;
  size_t sort_bytes;
  uint32_t* row_start;       // [grid_y + 1]
  uint32_t* chunk_first;     // [grid_y + 1]
  uint32_t* chunk_counts;    // [max_chunks][grid_x]
  uint32_t* tile_total;      // [tiles]
  uint32_t* tile_start;      // [tiles]
  void* scan_tmp;
  size_t scan_bytes;
  uint32_t max_chunks;
};

// Row pairs per chunk of the binning passes.
constexpr int kRowChunk = 2048;

uint32_t max_chunks(uint32_t m, int grid_y) {
  return m / uint32_t(kRowChunk) + uint32_t(grid_y) + 1u;
}

size_t pair_sort_bytes(uint32_t m) {
  size_t bytes = 0;
  cub::DeviceRadixSort::SortPairs(nullptr, bytes, (uint32_t*)nullptr, (uint32_t*)nullptr,
                                  (uint64_t*)nullptr, (uint64_t*)nullptr, int(m), 0, 32);
  return bytes;
}

size_t tile_scan_bytes(int tiles) {
  size_t bytes = 0;
  cub::DeviceScan::ExclusiveSum(nullptr, bytes, (uint32_t*)nullptr, (uint32_t*)nullptr, tiles);
  return bytes;
}

size_t binning_bytes(uint32_t n, uint32_t m, int grid_x, int grid_y) {
  const int tiles = grid_x * grid_y;
  return aligned<uint32_t>(4 * size_t(n)) + 2 * aligned<uint32_t>(4 * size_t(m)) +
         2 * aligned<uint64_t>(8 * size_t(m)) +
         aligned<char>(pair_sort_bytes(m)) + 2 * aligned<uint32_t>(4 * size_t(grid_y + 1)) +
         aligned<uint32_t>(4 * size_t(max_chunks(m, grid_y)) * grid_x) +
         2 * aligned<uint32_t>(4 * size_t(tiles)) + aligned<char>(tile_scan_bytes(tiles)) + 128;
}

uint32_t* point_list_from(const void* base) {
  return reinterpret_cast<uint32_t*>((reinterpret_cast<uintptr_t>(base) + 127) &
                                     ~uintptr_t(127));
}

BinningState binning_from(char* base, uint32_t n, uint32_t m, int grid_x, int grid_y) {
  BinningState b;
  const int tiles = grid_x * grid_y;
  char* c = reinterpret_cast<char*>(point_list_from(base));
  auto take = [&](size_t bytes) {
    char* r = c;
    c += aligned<char>(bytes);
    return r;
  };
  b.values = reinterpret_cast<uint32_t*>(take(4 * size_t(n)));
  b.pair_rows = reinterpret_cast<uint32_t*>(take(4 * size_t(m)));
  b.pair_rows_sorted = reinterpret_cast<uint32_t*>(take(4 * size_t(m)));
  b.pair_spans = reinterpret_cast<uint64_t*>(take(8 * size_t(m)));
  b.pair_spans_sorted = reinterpret_cast<uint64_t*>(take(8 * size_t(m)));
  b.sort_bytes = pair_sort_bytes(m);
  b.sort_tmp = take(b.sort_bytes);
  b.row_start = reinterpret_cast<uint32_t*>(take(4 * size_t(grid_y + 1)));
  b.chunk_first = reinterpret_cast<uint32_t*>(take(4 * size_t(grid_y + 1)));
  b.max_chunks = max_chunks(m, grid_y);
  b.chunk_counts = reinterpret_cast<uint32_t*>(take(4 * size_t(b.max_chunks) * grid_x));
  b.tile_total = reinterpret_cast<uint32_t*>(take(4 * size_t(tiles)));
  b.tile_start = reinterpret_cast<uint32_t*>(take(4 * size_t(tiles)));
  b.scan_bytes = tile_scan_bytes(tiles);
  b.scan_tmp = take(b.scan_bytes);
  return b;
}

struct Camera {
  const float* view;  // column-major 4x4
  const float* proj;  // column-major 4x4 (full projection)
  const float* campos;
  float tan_x, tan_y, fx, fy;
  int width, height, grid_x, grid_y;
};

// ---------------------------------------------------------------------------
// Forward kernels.

__global__ void preprocess_kernel(int P, const float* __restrict__ means,
                                  const float* __restrict__ scales, float scale_modifier,
                                  const float* __restrict__ rotations,
                                  const float* __restrict__ opacities,
                                  const float* __restrict__ colors_precomp,
                                  const float* __restrict__ cov3d_precomp, Camera cam,
                                  bool antialiasing, GeomState g,
                                  int* __restrict__ radii_out) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= P) return;
  g.radii[i] = 0;
  g.tiles[i] = 0;
  g.rows[i] = 0;
  radii_out[i] = 0;
  const Vec3 p{means[3 * i], means[3 * i + 1], means[3 * i + 2]};
  const Vec3 t = affine3(cam.view, p);
  if (t.z <= kNearPlane) return;
  float cov[6];
  if (cov3d_precomp) {
#pragma unroll
    for (int k = 0; k < 6; ++k) cov[k] = cov3d_precomp[6 * i + k];
  } else {
    const float s[3] = {scale_modifier * scales[3 * i], scale_modifier * scales[3 * i + 1],
                        scale_modifier * scales[3 * i + 2]};
    const float q[4] = {rotations[4 * i], rotations[4 * i + 1], rotations[4 * i + 2],
                        rotations[4 * i + 3]};
    covariance3d(s, q, cov);
  }
#pragma unroll
  for (int k = 0; k < 6; ++k) g.cov3d[6 * i + k] = cov[k];
  const Projection2 J = screen_jacobian(t, cam.fx, cam.fy, cam.tan_x, cam.tan_y, cam.view);
  float a, b, c;
  covariance2d(J, cov, a, b, c);
  const float det0 = a * c - b * b;
  a += kLowPass;
  c += kLowPass;
  const float det = a * c - b * b;
  float aa = 1.f;
  if (antialiasing) aa = sqrtf(fmaxf(0.000025f, det0 / det));
  if (det == 0.f) return;
  const float inv = 1.f / det;
  const float mid = 0.5f * (a + c);
  const float disc = sqrtf(fmaxf(0.1f, mid * mid - det));
  const float lambda = fmaxf(mid + disc, mid - disc);
  const int radius = (int)ceilf(3.f * sqrtf(lambda));
  const float hw = affine_w(cam.proj, p);
  const Vec3 h = affine3(cam.proj, p);
  const float iw = 1.f / (hw + 0.0000001f);
  const float px = ndc_to_pixel(h.x * iw, cam.width), py = ndc_to_pixel(h.y * iw, cam.height);
  int x0, y0, x1, y1;
  tile_rect(px, py, radius, cam.grid_x, cam.grid_y, x0, y0, x1, y1);
  const int touched = (x1 - x0) * (y1 - y0);
  if (touched == 0) return;
  // SH colours come from sh_colour_kernel (coalesced coefficient reads).
  // Given colours were clamped by whoever made them (if at all): no channel
  // is masked in the seeds taken from this view.
  if (colors_precomp) {
#pragma unroll
    for (int k = 0; k < 3; ++k) {
      g.rgb[3 * i + k] = colors_precomp[3 * i + k];
      g.clamped[3 * i + k] = false;
    }
  }
  g.depth[i] = t.z;
  g.radii[i] = radius;
  radii_out[i] = radius;
  g.mean2d[i] = make_float2(px, py);
  const float4 co = make_float4(c * inv, -b * inv, a * inv, opacities[i] * aa);
  g.conic_opacity[i] = co;
  // Instances only for the tiles some pixel of which the Gaussian can reach
  // (see Footprint); the radius and everything else keep the 3-sigma rule.
  const Footprint f = make_footprint(px, py, co, radius, cam.grid_x, cam.grid_y);
  const uint32_t n = footprint_tiles(f);
  g.tiles[i] = n;
  g.rows[i] = n ? uint32_t(f.y1 - f.y0) : 0u;
}

// Binning. Every tile's instance list is its Gaussians in depth order (ties by
// Gaussian index), which is what a stable sort of one (tile << 32 | depth) key
// per instance gives; here no per-instance key is sorted:
//  1. the Gaussians are ordered by depth (a stable sort of P depth keys);
//  2. each Gaussian, in depth order, writes one pair per row of its tile
//     rectangle: key = tile row, value = (Gaussian id, first and one-past-last
//     tile of its footprint in that row, see Footprint); the pairs are
//     stable-sorted by row (a 7-bit key at 1080p: one radix pass);
//  3. each row's pairs are cut into chunks of kRowChunk; a first pass counts
//     every chunk's instances per tile (difference array in shared memory);
//  4. per tile the chunk counts become chunk offsets and the tile totals are
//     scanned into tile starts (and the ranges);
//  5. a second pass ranks each chunk's instances within their tiles from lane
//     masks of the pairs covering each tile (pair order kept) and writes every
//     tile's run of Gaussian ids contiguously.
constexpr int kBinThreads = 256;

__device__ __forceinline__ uint64_t pack_pair(uint32_t id, int lo, int hi) {
  return uint64_t(id) | (uint64_t(uint32_t(lo)) << 32) | (uint64_t(uint32_t(hi)) << 48);
}

__global__ void depth_key_kernel(int P, GeomState g) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= P) return;
  // Depths of drawn Gaussians are positive, so their bits order like floats;
  // Gaussians without tiles go last.
  g.depth_keys[i] = g.tiles[i] > 0 ? __float_as_uint(g.depth[i]) : 0xffffffffu;
  g.ids[i] = uint32_t(i);
}

// Tile-rectangle rows of the Gaussians in depth order (to be scanned).
__global__ void gather_rows_kernel(int P, GeomState g) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= P) return;
  g.depth_keys[i] = g.rows[g.order[i]];
}

// A warp per 32 Gaussians in depth order: each lane builds one Gaussian's
// footprint in shared memory, then the warp walks the 32 Gaussians' pairs
// together, one pair per lane (the owner found by a search of the warp's pair
// offsets). The Gaussians' pairs are consecutive in depth order, so the stores
// are contiguous and no lane waits for a Gaussian with many rows. (Emitting in
// Gaussian-id order, with coalesced reads but scattered writes, was slower.)
constexpr int kEmitWarps = 8;

__global__ void __launch_bounds__(32 * kEmitWarps)
    emit_rows_kernel(int P, GeomState g, int grid_x, int grid_y,
                     uint32_t* __restrict__ rows_out, uint64_t* __restrict__ spans_out) {
  __shared__ Footprint s_fp[kEmitWarps][32];
  __shared__ uint32_t s_id[kEmitWarps][32];
  __shared__ uint32_t s_first[kEmitWarps][33];  // first pair of each lane's Gaussian; [32]: total
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int i0 = (blockIdx.x * kEmitWarps + warp) * 32;
  if (i0 >= P) return;  // whole warp
  const int i = i0 + lane;
  uint32_t n = 0;
  if (i < P) {
    const uint32_t id = g.order[i];
    n = g.rows[id];
    if (n) {
      const float2 m = g.mean2d[id];
      s_fp[warp][lane] = make_footprint(m.x, m.y, g.conic_opacity[id], g.radii[id], grid_x,
                                        grid_y);
    }
    s_id[warp][lane] = id;
  }
  uint32_t inc = n;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const uint32_t t = __shfl_up_sync(0xffffffffu, inc, o);
    if (lane >= o) inc += t;
  }
  s_first[warp][lane] = inc - n;
  if (lane == 31) s_first[warp][32] = inc;
  const uint32_t base = i0 == 0 ? 0u : g.offsets[i0 - 1];  // the warp's first pair
  __syncwarp();
  const uint32_t total = s_first[warp][32];
  for (uint32_t j = lane; j < total; j += 32) {
    // Owner: the last lane whose first pair is at or before j (a lane without
    // pairs shares its successor's first pair, so the last one has pairs).
    int lo = 0, hi = 31;
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (s_first[warp][mid] <= j) lo = mid;
      else hi = mid - 1;
    }
    const Footprint& f = s_fp[warp][lo];
    const int ty = f.y0 + int(j - s_first[warp][lo]);
    int x_lo, x_hi;
    row_span(f, ty, x_lo, x_hi);
    if (x_hi < x_lo) x_hi = x_lo;
    rows_out[base + j] = uint32_t(ty);
    spans_out[base + j] = pack_pair(s_id[warp][lo], x_lo, x_hi);
  }
}

__device__ __forceinline__ uint32_t lower_bound(const uint32_t* keys, uint32_t n,
                                                uint32_t value) {
  uint32_t lo = 0, hi = n;
  while (lo < hi) {
    const uint32_t mid = lo + (hi - lo) / 2;
    if (keys[mid] < value) lo = mid + 1;
    else hi = mid;
  }
  return lo;
}

// First pair of every tile row (row_start[grid_y] = m) and the first chunk of
// every row (chunk_first[grid_y] = number of chunks). One block.
__global__ void row_layout_kernel(uint32_t m, int grid_y, const uint32_t* __restrict__ rows,
                                  uint32_t* __restrict__ row_start,
                                  uint32_t* __restrict__ chunk_first) {
  for (int ty = threadIdx.x; ty <= grid_y; ty += blockDim.x)
    row_start[ty] = ty == grid_y ? m : lower_bound(rows, m, uint32_t(ty));
  __syncthreads();
  if (threadIdx.x == 0) {
    uint32_t c = 0;
    for (int ty = 0; ty < grid_y; ++ty) {
      chunk_first[ty] = c;
      c += (row_start[ty + 1] - row_start[ty] + kRowChunk - 1) / kRowChunk;
    }
    chunk_first[grid_y] = c;
  }
}

// The tile row of chunk c: the last row whose first chunk is <= c.
__device__ __forceinline__ int chunk_row(const uint32_t* chunk_first, int grid_y, uint32_t c) {
  int lo = 0, hi = grid_y - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) / 2;
    if (chunk_first[mid] <= c) lo = mid;
    else hi = mid - 1;
  }
  return lo;
}

__global__ void __launch_bounds__(kBinThreads)
    tile_count_kernel(int grid_x, int grid_y, const uint64_t* __restrict__ spans,
                      const uint32_t* __restrict__ row_start,
                      const uint32_t* __restrict__ chunk_first,
                      uint32_t* __restrict__ chunk_counts) {
  extern __shared__ int diff[];  // grid_x + 1
  const uint32_t c = blockIdx.x;
  if (c >= chunk_first[grid_y]) return;  // whole block
  const int ty = chunk_row(chunk_first, grid_y, c);
  const uint32_t begin = row_start[ty] + (c - chunk_first[ty]) * kRowChunk;
  const uint32_t end = min(row_start[ty + 1], begin + kRowChunk);
  for (int x = threadIdx.x; x <= grid_x; x += blockDim.x) diff[x] = 0;
  __syncthreads();
  for (uint32_t p = begin + threadIdx.x; p < end; p += blockDim.x) {
    const uint64_t v = spans[p];
    const int lo = int((v >> 32) & 0xffffu), hi = int(v >> 48);
    if (hi > lo) {
      atomicAdd(&diff[lo], 1);
      atomicAdd(&diff[hi], -1);
    }
  }
  __syncthreads();
  if (threadIdx.x < 32) {  // inclusive scan of the differences, 32 tiles at a time
    const int lane = threadIdx.x;
    int carry = 0;
    for (int x0 = 0; x0 < grid_x; x0 += 32) {
      const int x = x0 + lane;
      int v = x < grid_x ? diff[x] : 0;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int t = __shfl_up_sync(0xffffffffu, v, o);
        if (lane >= o) v += t;
      }
      if (x < grid_x) chunk_counts[size_t(c) * grid_x + x] = uint32_t(carry + v);
      carry += __shfl_sync(0xffffffffu, v, 31);
    }
  }
}

// Per tile: chunk counts -> offsets of each chunk within the tile, and the total.
// A block takes one tile row and 32 tiles (lane = tile); the row's chunks are
// split into one contiguous segment per warp, each warp sums its segment, and
// after the segment sums are known each warp rewrites its counts as offsets.
constexpr int kBinWarps = kBinThreads / 32;

__global__ void __launch_bounds__(kBinThreads)
    tile_totals_kernel(int grid_x, const uint32_t* __restrict__ chunk_first,
                       uint32_t* __restrict__ chunk_counts, uint32_t* __restrict__ tile_total) {
  __shared__ uint32_t segment[kBinWarps][32];
  const int ty = blockIdx.y, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int x = blockIdx.x * 32 + lane;
  const uint32_t c0 = chunk_first[ty], chunks = chunk_first[ty + 1] - c0;
  const uint32_t per = (chunks + kBinWarps - 1) / kBinWarps;
  const uint32_t a = c0 + min(chunks, uint32_t(warp) * per);
  const uint32_t e = c0 + min(chunks, uint32_t(warp + 1) * per);
  uint32_t sum = 0;
  if (x < grid_x)
    for (uint32_t c = a; c < e; ++c) sum += chunk_counts[size_t(c) * grid_x + x];
  segment[warp][lane] = sum;
  __syncthreads();
  if (x >= grid_x) return;
  uint32_t running = 0;
  for (int w = 0; w < warp; ++w) running += segment[w][lane];
  for (uint32_t c = a; c < e; ++c) {
    const uint32_t v = chunk_counts[size_t(c) * grid_x + x];
    chunk_counts[size_t(c) * grid_x + x] = running;
    running += v;
  }
  if (warp == kBinWarps - 1) tile_total[ty * grid_x + x] = running;
}

__global__ void tile_ranges_kernel(int tiles, const uint32_t* __restrict__ tile_start,
                                   const uint32_t* __restrict__ tile_total,
                                   uint2* __restrict__ ranges) {
  const int t = blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= tiles) return;
  ranges[t] = make_uint2(tile_start[t], tile_start[t] + tile_total[t]);
}

// Second pass: per chunk, rounds of 256 pairs (one pair per thread, 32 per
// warp). Each warp marks its pairs' spans in a per-tile lane mask (the XOR of a
// lane bit at lo and at hi, prefix-XORed across the tiles gives, for every tile,
// the lanes whose span covers it), so an instance's slot is its tile's next free
// slot plus the instances of that tile in earlier warps of the round plus the
// popcount of the earlier lanes in its warp's mask: pair order (= depth order)
// is kept within every tile.
__host__ __device__ constexpr int cover_index(int x) { return x + (x >> 5); }  // bank skew

size_t place_shared_bytes(int grid_x) {
  return sizeof(uint32_t) * (size_t(kBinWarps) * (cover_index(grid_x) + 1) +
                             size_t(kBinWarps) * grid_x + size_t(grid_x));
}

__global__ void __launch_bounds__(kBinThreads)
    place_kernel(int grid_x, int grid_y, uint32_t n, const uint64_t* __restrict__ spans,
                 const uint32_t* __restrict__ row_start,
                 const uint32_t* __restrict__ chunk_first,
                 const uint32_t* __restrict__ chunk_offsets,
                 const uint32_t* __restrict__ tile_start, uint32_t* __restrict__ values) {
  extern __shared__ uint32_t dyn[];
  const int G = grid_x, stride = cover_index(G) + 1;
  uint32_t* cover_all = dyn;                       // [warps][cover_index(G) + 1] lane masks
  uint32_t* slot_all = cover_all + kBinWarps * stride;  // [warps][G] first slot of the warp
  uint32_t* next = slot_all + kBinWarps * G;       // [G] the tile's next free slot
  const uint32_t c = blockIdx.x;
  if (c >= chunk_first[grid_y]) return;  // whole block
  const int ty = chunk_row(chunk_first, grid_y, c);
  const uint32_t begin = row_start[ty] + (c - chunk_first[ty]) * kRowChunk;
  const uint32_t count = min(row_start[ty + 1], begin + kRowChunk) - begin;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  uint32_t* cover = cover_all + warp * stride;
  const uint32_t* slot = slot_all + warp * G;
  for (int x = threadIdx.x; x < kBinWarps * stride; x += kBinThreads) cover_all[x] = 0;
  for (int x = threadIdx.x; x < G; x += kBinThreads)
    next[x] = tile_start[ty * G + x] + chunk_offsets[size_t(c) * G + x];
  // Each lane prefix-XORs a contiguous run of tiles.
  const int per = (G + 31) / 32;
  const int s0 = min(G, lane * per), s1 = min(G, s0 + per);
  const uint32_t bit = 1u << lane, earlier = bit - 1u;
  for (uint32_t r0 = 0; r0 < count; r0 += kBinThreads) {  // the same trips everywhere
    __syncthreads();  // the previous round's shared state consumed
    const uint32_t p = r0 + threadIdx.x;
    uint32_t id = 0, lo = 0, hi = 0;
    if (p < count) {
      const uint64_t v = spans[begin + p];
      id = uint32_t(v);
      hi = min(uint32_t(v >> 48), uint32_t(G));
      lo = min(uint32_t(v >> 32) & 0xffffu, hi);
    }
    if (hi > lo) {
      atomicXor(&cover[cover_index(lo)], bit);
      atomicXor(&cover[cover_index(hi)], bit);
    }
    __syncwarp();
    uint32_t acc = 0;
    for (int x = s0; x < s1; ++x) acc ^= cover[cover_index(x)];
    uint32_t inc = acc;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const uint32_t t = __shfl_up_sync(0xffffffffu, inc, o);
      if (lane >= o) inc ^= t;
    }
    uint32_t run = inc ^ acc;
    for (int x = s0; x < s1; ++x) {
      run ^= cover[cover_index(x)];
      cover[cover_index(x)] = run;
    }
    __syncthreads();  // every warp's masks ready
    for (int x = threadIdx.x; x < G; x += kBinThreads) {
      uint32_t at = next[x];
      for (int w = 0; w < kBinWarps; ++w) {
        slot_all[w * G + x] = at;
        at += __popc(cover_all[w * stride + cover_index(x)]);
      }
      next[x] = at;
    }
    __syncthreads();  // slots ready
    for (uint32_t x = lo; x < hi; ++x) {
      const uint32_t pos = slot[x] + __popc(cover[cover_index(x)] & earlier);
      if (pos < n) values[pos] = id;
    }
    __syncwarp();  // the warp's masks used
    for (int x = lane; x < stride; x += 32) cover[x] = 0;
  }
}

__global__ void __launch_bounds__(kTilePixels)
    render_forward_kernel(const uint2* __restrict__ ranges,
                          const uint32_t* __restrict__ point_list, int width, int height,
                          int grid_x, const float2* __restrict__ mean2d,
                          const float* __restrict__ rgb,
                          const float4* __restrict__ conic_opacity,
                          const float* __restrict__ depth, const float* __restrict__ bg,
                          float* __restrict__ final_t, uint32_t* __restrict__ n_contrib,
                          float* __restrict__ out_color, float* __restrict__ out_invdepth) {
  const int tile = blockIdx.y * grid_x + blockIdx.x;
  const int px = blockIdx.x * kTileX + threadIdx.x % kTileX;
  const int py = blockIdx.y * kTileY + threadIdx.x / kTileX;
  const bool inside = px < width && py < height;
  const int pix = py * width + px;
  const float fx = (float)px, fy = (float)py;
  const uint2 range = ranges[tile];
  __shared__ float2 s_xy[kBatch];
  __shared__ float4 s_co[kBatch];
  __shared__ float s_rgb[3 * kBatch];
  __shared__ float s_inv[kBatch];
  bool done = !inside;
  float T = 1.f, C[3] = {0.f, 0.f, 0.f}, D = 0.f;
  uint32_t contributor = 0, last = 0;
  const int todo = int(range.y - range.x);
  for (int base = 0; base < todo; base += kBatch) {
    if (__syncthreads_count(done) == kTilePixels) break;
    const int k = base + threadIdx.x;
    if (k < todo) {
      const uint32_t id = point_list[range.x + k];
      s_xy[threadIdx.x] = mean2d[id];
      s_co[threadIdx.x] = conic_opacity[id];
      s_rgb[3 * threadIdx.x] = rgb[3 * id];
      s_rgb[3 * threadIdx.x + 1] = rgb[3 * id + 1];
      s_rgb[3 * threadIdx.x + 2] = rgb[3 * id + 2];
      s_inv[threadIdx.x] = 1.f / depth[id];
    }
    __syncthreads();
    const int count = min(kBatch, todo - base);
    for (int j = 0; !done && j < count; ++j) {
      ++contributor;
      const float dx = s_xy[j].x - fx, dy = s_xy[j].y - fy;
      const float4 co = s_co[j];
      const float power = gauss_power(co, dx, dy);
      if (power > 0.f) continue;
      const float alpha = fminf(kMaxAlpha, co.w * __expf(power));
      if (alpha < kMinAlpha) continue;
      const float test_t = T * (1.f - alpha);
      if (test_t < kMinTransmittance) {
        done = true;
        continue;
      }
      const float w = alpha * T;
      C[0] += s_rgb[3 * j] * w;
      C[1] += s_rgb[3 * j + 1] * w;
      C[2] += s_rgb[3 * j + 2] * w;
      D += s_inv[j] * w;
      T = test_t;
      last = contributor;
    }
  }
  if (inside) {
    final_t[pix] = T;
    n_contrib[pix] = last;
    const int hw = width * height;
    out_color[pix] = C[0] + T * bg[0];
    out_color[hw + pix] = C[1] + T * bg[1];
    out_color[2 * hw + pix] = C[2] + T * bg[2];
    if (out_invdepth) out_invdepth[pix] = D;
  }
}

// ---------------------------------------------------------------------------
// Pixel backward (the algebra, warp reductions and field slots are in
// raster_adjoint.cuh).

struct PixelGrads {
  float* dmean2d;    // [P][3]
  float* dconic;     // [P][4] (a, b, -, c)
  float* dopacity;   // [P]
  float* dcolor;     // [P][3]
  float* dinvdepth;  // [P] or null
};

// Address of adjoint field f (Field slots) of Gaussian id.
__device__ __forceinline__ float* field_address(const PixelGrads& o, uint32_t id, int f) {
  switch (f) {
    case kRed: case kGreen: case kBlue: return o.dcolor + 3 * size_t(id) + f;
    case kMeanX: case kMeanY: return o.dmean2d + 3 * size_t(id) + (f - kMeanX);
    case kConicA: return o.dconic + 4 * size_t(id);
    case kConicB: return o.dconic + 4 * size_t(id) + 1;
    case kConicC: return o.dconic + 4 * size_t(id) + 3;
    case kOpacity: return o.dopacity + id;
    default: return o.dinvdepth + id;
  }
}

// Shared-memory batch of Gaussians of one tile, staged back to front.
struct TileBatch {
  uint32_t id[kBatch];
  float2 xy[kBatch];
  float4 co[kBatch];
  float rgb[3 * kBatch];
  float inv[kBatch];
};

// Loads slot `slot` of the batch starting `base` Gaussians from the back of
// the first `todo` entries of the tile's list.
__device__ __forceinline__ void stage_back_to_front(TileBatch& s, int slot, int base, int todo,
                                                    uint2 range,
                                                    const uint32_t* __restrict__ point_list,
                                                    const float2* __restrict__ mean2d,
                                                    const float4* __restrict__ conic_opacity,
                                                    const float* __restrict__ rgb,
                                                    const float* __restrict__ depth) {
  const int k = base + slot;
  if (k >= todo) return;
  const uint32_t id = point_list[range.x + todo - k - 1];
  s.id[slot] = id;
  s.xy[slot] = mean2d[id];
  s.co[slot] = conic_opacity[id];
  s.rgb[3 * slot] = rgb[3 * id];
  s.rgb[3 * slot + 1] = rgb[3 * id + 1];
  s.rgb[3 * slot + 2] = rgb[3 * id + 2];
  s.inv[slot] = 1.f / depth[id];
}

// Largest last-contributor count over the block's pixels: no pixel of the
// tile has a contributor past it, so the walk starts there instead of at the
// end of the tile's list (the Gaussians skipped contribute nothing).
__device__ __forceinline__ int block_walk_length(uint32_t my_last, uint32_t* s_max) {
  if (threadIdx.x == 0) *s_max = 0;
  __syncthreads();
  const uint32_t warp_max = __reduce_max_sync(0xffffffffu, my_last);
  if ((threadIdx.x & 31) == 0) atomicMax(s_max, warp_max);
  __syncthreads();
  return int(*s_max);
}

// Modes 0 and 1, one pixel per thread (mode 2 is render_backward_pairs_kernel).
template <int Mode>
__global__ void __launch_bounds__(kTilePixels)
    render_backward_kernel(const uint2* __restrict__ ranges,
                           const uint32_t* __restrict__ point_list, int width, int height,
                           int grid_x, const float* __restrict__ bg,
                           const float2* __restrict__ mean2d,
                           const float4* __restrict__ conic_opacity,
                           const float* __restrict__ rgb, const float* __restrict__ depth,
                           const float* __restrict__ final_t,
                           const uint32_t* __restrict__ n_contrib,
                           const float* __restrict__ dpixels,
                           const float* __restrict__ dinvdepth_pixels, PixelGrads out) {
  const int tile = blockIdx.y * grid_x + blockIdx.x;
  const int px = blockIdx.x * kTileX + threadIdx.x % kTileX;
  const int py = blockIdx.y * kTileY + threadIdx.x / kTileX;
  const int lane = threadIdx.x & 31;
  const uint2 range = ranges[tile];
  __shared__ TileBatch s;
  __shared__ uint32_t s_max;
  PixelWalk pixel;
  walk_begin(pixel, px, py, width, height, final_t, n_contrib, dpixels, dinvdepth_pixels, bg);
  const int todo = block_walk_length(pixel.last, &s_max);
  const float fx = (float)px, fy = (float)py;
  const float half_w = 0.5f * width, half_h = 0.5f * height;
  const int fields = out.dinvdepth ? kFields : kFields - 1;
  for (int base = 0; base < todo; base += kBatch) {
    __syncthreads();
    stage_back_to_front(s, threadIdx.x, base, todo, range, point_list, mean2d, conic_opacity,
                        rgb, depth);
    __syncthreads();
    const int count = min(kBatch, todo - base);
    for (int j = 0; j < count; ++j) {
      float f[16];
#pragma unroll
      for (int q = 0; q < 16; ++q) f[q] = 0.f;
      const float4 co = s.co[j];
      const uint32_t index = uint32_t(todo - 1 - (base + j));
      const float dx = s.xy[j].x - fx, dy = s.xy[j].y - fy;
      if (!walk_step(pixel, index, gauss_power(co, dx, dy), dx, dy, co, s.rgb + 3 * j,
                     s.inv[j], f))
        continue;
      finish_moments(f, co, half_w, half_h);
      const uint32_t id = s.id[j];
      auto dest = [&](int q) { return field_address(out, id, q); };
      if constexpr (Mode == 0) {
        for (int q = 0; q < fields; ++q) atomicAdd(dest(q), f[q]);
      } else {
        accumulate_by_key(id, f, fields, lane, dest);
      }
    }
  }
}

// Mode 2 with kPixelsPerThread pixels per thread: rows y, y + 16/k, ... of the
// tile. Per Gaussian a thread adds its pixels' moments first, so each warp
// reduction covers 32 k pixels.
#ifndef CLAD3DGS_PIXELS_PER_THREAD
#define CLAD3DGS_PIXELS_PER_THREAD 4
#endif
constexpr int kPixelsPerThread = CLAD3DGS_PIXELS_PER_THREAD;
constexpr int kPairThreads = kTilePixels / kPixelsPerThread;
constexpr int kRowStep = kTileY / kPixelsPerThread;

// Twelve resident 64-thread blocks per SM (at most 85 registers a thread): the
// measured best at 1080p/3M (1.30 ms against 1.43 ms unconstrained at 93
// registers and 1.37 ms at 64).
#ifndef CLAD3DGS_PAIR_MIN_BLOCKS
#define CLAD3DGS_PAIR_MIN_BLOCKS 12
#endif
__global__ void __launch_bounds__(kPairThreads, CLAD3DGS_PAIR_MIN_BLOCKS)
    render_backward_pairs_kernel(const uint2* __restrict__ ranges,
                                 const uint32_t* __restrict__ point_list, int width,
                                 int height, int grid_x, const float* __restrict__ bg,
                                 const float2* __restrict__ mean2d,
                                 const float4* __restrict__ conic_opacity,
                                 const float* __restrict__ rgb, const float* __restrict__ depth,
                                 const float* __restrict__ final_t,
                                 const uint32_t* __restrict__ n_contrib,
                                 const float* __restrict__ dpixels,
                                 const float* __restrict__ dinvdepth_pixels, PixelGrads out) {
  const int tile = blockIdx.y * grid_x + blockIdx.x;
  const int px = blockIdx.x * kTileX + threadIdx.x % kTileX;
  const int py = blockIdx.y * kTileY + threadIdx.x / kTileX;  // first row of this thread
  const int lane = threadIdx.x & 31;
  const uint2 range = ranges[tile];
  __shared__ TileBatch s;
  __shared__ uint32_t s_max;
  PixelWalk pixel[kPixelsPerThread];
  uint32_t my_last = 0;
#pragma unroll
  for (int r = 0; r < kPixelsPerThread; ++r) {
    walk_begin(pixel[r], px, py + r * kRowStep, width, height, final_t, n_contrib, dpixels,
               dinvdepth_pixels, bg);
    my_last = max(my_last, pixel[r].last);
  }
  const int todo = block_walk_length(my_last, &s_max);
  const float fx = (float)px;
  const float half_w = 0.5f * width, half_h = 0.5f * height;
  const int fields = out.dinvdepth ? kFields : kFields - 1;
  for (int base = 0; base < todo; base += kBatch) {
    __syncthreads();
#pragma unroll
    for (int h = 0; h < kPixelsPerThread; ++h)
      stage_back_to_front(s, threadIdx.x + h * kPairThreads, base, todo, range, point_list,
                          mean2d, conic_opacity, rgb, depth);
    __syncthreads();
    const int count = min(kBatch, todo - base);
    for (int j = 0; j < count; ++j) {
      float f[16];
#pragma unroll
      for (int q = 0; q < 16; ++q) f[q] = 0.f;
      const float2 xy = s.xy[j];
      const float4 co = s.co[j];
      const uint32_t index = uint32_t(todo - 1 - (base + j));
      const float dx = xy.x - fx;
      const ColumnForm column = column_form(co, dx);
      bool any = false;
#pragma unroll
      for (int r = 0; r < kPixelsPerThread; ++r) {
        const float dy = xy.y - (float)(py + r * kRowStep);
        any = walk_step(pixel[r], index, row_power(column, dy), dx, dy, co, s.rgb + 3 * j,
                        s.inv[j], f) || any;
      }
      if (!__any_sync(0xffffffffu, any)) continue;
      finish_moments(f, co, half_w, half_h);
      const uint32_t id = s.id[j];
      accumulate_converged(f, fields, lane, [&](int q) { return field_address(out, id, q); });
    }
  }
}

// Counting pass of the pixel backward (not part of it): replays the walk's
// contribution test, one pixel per thread in the 256-thread layout of modes 0
// and 1, and tallies per tile
//   counts[0] contributing (pixel, Gaussian) pairs (mode 0 issues one atomic
//             per pair and field);
//   counts[1] mode 1's atomics per field: per (warp, Gaussian) 1 when all 32
//             lanes contribute, else the contributing lanes;
//   counts[2] mode 2's warp reductions (one 9- or 10-lane atomic instruction
//             each): per (warp of the four-pixels-per-thread layout, Gaussian)
//             with any contributing lane. That warp holds pixel rows
//             {0,1,4,5,8,9,12,13} (warp 0) or {2,3,6,7,10,11,14,15} (warp 1)
//             of the tile, i.e. the one-pixel warps w with w % 2 equal to it.
__global__ void __launch_bounds__(kTilePixels)
    count_accumulation_kernel(const uint2* __restrict__ ranges,
                              const uint32_t* __restrict__ point_list, int width, int height,
                              int grid_x, const float2* __restrict__ mean2d,
                              const float4* __restrict__ conic_opacity,
                              const uint32_t* __restrict__ n_contrib,
                              unsigned long long* __restrict__ counts) {
  static_assert(kTilePixels == 256 && kPixelsPerThread == 4, "counting layout");
  const int tile = blockIdx.y * grid_x + blockIdx.x;
  const int px = blockIdx.x * kTileX + threadIdx.x % kTileX;
  const int py = blockIdx.y * kTileY + threadIdx.x / kTileX;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const bool inside = px < width && py < height;
  const uint32_t last = inside ? n_contrib[py * width + px] : 0;
  const uint2 range = ranges[tile];
  __shared__ uint32_t s_max;
  __shared__ float2 s_xy[kBatch];
  __shared__ float4 s_co[kBatch];
  __shared__ unsigned char s_any[kBatch][8];  // per Gaussian of the batch and warp
  const int todo = block_walk_length(last, &s_max);
  const float fx = (float)px, fy = (float)py;
  unsigned long long pairs = 0, whole_or_lanes = 0, reductions = 0;
  for (int base = 0; base < todo; base += kBatch) {
    __syncthreads();
    const int k = base + threadIdx.x;
    if (k < todo) {
      const uint32_t id = point_list[range.x + todo - k - 1];
      s_xy[threadIdx.x] = mean2d[id];
      s_co[threadIdx.x] = conic_opacity[id];
    }
    __syncthreads();
    const int count = min(kBatch, todo - base);
    for (int j = 0; j < count; ++j) {
      const uint32_t index = uint32_t(todo - 1 - (base + j));
      const float4 co = s_co[j];
      const float p = gauss_power(co, s_xy[j].x - fx, s_xy[j].y - fy);
      const float alpha = fminf(kMaxAlpha, co.w * __expf(p));
      const bool live = index < last && p <= 0.f && alpha >= kMinAlpha;
      const unsigned lanes = __ballot_sync(0xffffffffu, live);
      if (lane == 0) {
        pairs += __popc(lanes);
        whole_or_lanes += lanes == 0xffffffffu ? 1u : __popc(lanes);
        s_any[j][warp] = lanes != 0u;
      }
    }
    __syncthreads();
    if (threadIdx.x < count) {
      const unsigned char* a = s_any[threadIdx.x];
      reductions += (a[0] | a[2] | a[4] | a[6]) + (a[1] | a[3] | a[5] | a[7]);
    }
  }
  if (lane == 0 && (pairs || whole_or_lanes)) {
    atomicAdd(counts, pairs);
    atomicAdd(counts + 1, whole_or_lanes);
  }
  if (reductions) atomicAdd(counts + 2, reductions);
}

// Test probe of the accumulation helpers above on caller-given lane streams:
// thread i (linear index over the grid, blocks of whole warps) holds key[i],
// active[i] and values[i][0..fields). Mode 0: per-lane atomics; mode 1:
// accumulate_by_key (the pixel backward's mode 1); mode 2:
// accumulate_converged with every lane of the warp taking part and lanes that
// are inactive or past n adding zeros (keys must be the same for all lanes of
// a warp; a lane that disagrees records -1 in grouped[i] and its warp adds
// nothing). grouped[i] records whether lane i's values went through a warp
// reduction. Keys outside [0, rows) record -2 and add nothing.
__global__ void warp_probe_kernel(int mode, int n, int fields, const int* __restrict__ keys,
                                  const unsigned char* __restrict__ active,
                                  const float* __restrict__ values, float* __restrict__ out,
                                  int rows, int* __restrict__ grouped) {
  const int in_block = (threadIdx.z * blockDim.y + threadIdx.y) * blockDim.x + threadIdx.x;
  const int i = blockIdx.x * blockDim.x * blockDim.y * blockDim.z + in_block;
  const int lane = in_block & 31;
  if (mode == 2) {
    const bool in_range = i < n;
    const unsigned lanes = __ballot_sync(0xffffffffu, in_range);
    if (lanes == 0u) return;  // the whole warp is past n
    const int mine = in_range ? keys[i] : 0;
    const int key = __shfl_sync(0xffffffffu, mine, __ffs(lanes) - 1);
    const bool agree = __all_sync(0xffffffffu, !in_range || mine == key);
    const bool valid = key >= 0 && key < rows;
    if (!agree || !valid) {
      if (in_range) grouped[i] = agree ? -2 : -1;
      return;  // warp-uniform
    }
    float v[16];
#pragma unroll
    for (int q = 0; q < 16; ++q)
      v[q] = (in_range && active[i] && q < fields) ? values[size_t(i) * fields + q] : 0.f;
    if (in_range) grouped[i] = 1;
    accumulate_converged(v, fields, lane,
                         [&](int q) { return out + size_t(key) * fields + q; });
    return;
  }
  if (i >= n || !active[i]) return;
  const int key = keys[i];
  if (key < 0 || key >= rows) {
    grouped[i] = -2;
    return;
  }
  float v[16];
  for (int q = 0; q < fields; ++q) v[q] = values[size_t(i) * fields + q];
  auto dest = [&](int q) { return out + size_t(key) * fields + q; };
  if (mode == 1) {
    grouped[i] = whole_warp_on(uint32_t(key));
    accumulate_by_key(uint32_t(key), v, fields, lane, dest);
  } else {
    grouped[i] = 0;
    for (int q = 0; q < fields; ++q) atomicAdd(dest(q), v[q]);
  }
}

// ---------------------------------------------------------------------------
// Geometry backward: one thread per Gaussian (algebra in raster_adjoint.cuh).

struct GeomGrads {
  const float* dmean2d;    // [P][3]
  const float* dconic;     // [P][4]
  float* dopacity;         // [P] in: w.r.t. scaled opacity; out: w.r.t. opacity
  const float* dinvdepth;  // [P] or null
  float* dmeans;           // [P][3] out
  float* dcov3d;           // [P][6] out
  float* dscales;          // [P][3] out
  float* drotations;       // [P][4] out
};

__global__ void preprocess_backward_kernel(
    int P, const float* __restrict__ means, const float* __restrict__ scales,
    float scale_modifier, const float* __restrict__ rotations,
    const float* __restrict__ opacities, const float* __restrict__ cov3d_precomp, Camera cam,
    bool antialiasing, const int* __restrict__ radii, GeomState g, GeomGrads o) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= P) return;
  if (radii[i] <= 0) {
    // Outputs this kernel writes outright are zero for invisible Gaussians
    // (dmeans, accumulated with +=, and dopacity are left to the caller).
#pragma unroll
    for (int k = 0; k < 6; ++k) o.dcov3d[6 * i + k] = 0.f;
    if (!cov3d_precomp) {
#pragma unroll
      for (int k = 0; k < 3; ++k) o.dscales[3 * i + k] = 0.f;
#pragma unroll
      for (int k = 0; k < 4; ++k) o.drotations[4 * i + k] = 0.f;
    }
    return;
  }
  const Vec3 p{means[3 * i], means[3 * i + 1], means[3 * i + 2]};
  const Vec3 t = affine3(cam.view, p);
  const float* cov = g.cov3d + 6 * i;
  const Projection2 J = screen_jacobian(t, cam.fx, cam.fy, cam.tan_x, cam.tan_y, cam.view);
  const float* A0 = J.A;      // rows of A = J W
  const float* A1 = J.A + 3;
  // Screen covariance S2 (low-pass included) and the conic Q = S2^-1 of the forward.
  float a0, b, c0;
  covariance2d(J, cov, a0, b, c0);
  const Sym2 S2{a0 + kLowPass, b, c0 + kLowPass};
  const float det = S2.xx * S2.yy - b * b;
  const Sym2 Q{S2.yy / det, -b / det, S2.xx / det};
  // dL/dS2 = -Q Gq Q.
  const float* dq = o.dconic + 4 * i;
  const Sym2 QGQ = sandwich2(Q, Sym2{dq[0], dq[1], dq[3]});
  Sym2 Gs{-QGQ.xx, -QGQ.xy, -QGQ.yy};
  // Antialiasing scaled the opacity by s = sqrt(max(2.5e-5, r)),
  // r = det(S2 - 0.3 I) / det(S2).
  if (antialiasing) {
    const float dop_scaled = o.dopacity[i];
    const float det0 = a0 * c0 - b * b;
    const float r = det0 / det;
    const float s = sqrtf(fmaxf(0.000025f, r));
    o.dopacity[i] = dop_scaled * s;
    if (r > 0.000025f) {
      const float dr = dop_scaled * opacities[i] * 0.5f / s;
      const float k0 = dr / det, k1 = dr * det0 / (det * det);
      Gs.xx += k0 * c0 - k1 * S2.yy;
      Gs.xy -= (k0 - k1) * b;
      Gs.yy += k0 * a0 - k1 * S2.xx;
    }
  }
  // Gs A (2 x 3) serves both adjoints of the congruence S2 = A S3 A^T.
  float GA0[3], GA1[3];
#pragma unroll
  for (int c = 0; c < 3; ++c) {
    GA0[c] = Gs.xx * A0[c] + Gs.xy * A1[c];
    GA1[c] = Gs.xy * A0[c] + Gs.yy * A1[c];
  }
  // dL/dS3 = A^T Gs A, symmetric; stored as the upper triangle with the
  // off-diagonals counted for both positions.
  float G3[9];
#pragma unroll
  for (int r = 0; r < 3; ++r)
#pragma unroll
    for (int c = 0; c < 3; ++c) G3[3 * r + c] = A0[r] * GA0[c] + A1[r] * GA1[c];
  o.dcov3d[6 * i + 0] = G3[0];
  o.dcov3d[6 * i + 1] = 2.f * G3[1];
  o.dcov3d[6 * i + 2] = 2.f * G3[2];
  o.dcov3d[6 * i + 3] = G3[4];
  o.dcov3d[6 * i + 4] = 2.f * G3[5];
  o.dcov3d[6 * i + 5] = G3[8];
  // dL/dA = 2 Gs A S3.
  float S3[9];
  full3(cov, S3);
  float dA0[3], dA1[3];
#pragma unroll
  for (int c = 0; c < 3; ++c) {
    dA0[c] = 2.f * (GA0[0] * S3[c] + GA0[1] * S3[3 + c] + GA0[2] * S3[6 + c]);
    dA1[c] = 2.f * (GA1[0] * S3[c] + GA1[1] * S3[3 + c] + GA1[2] * S3[6 + c]);
  }
  // A = J W with W[k][c] = view[4c + k]: dL/dJ = dL/dA W^T. J's varying
  // entries: J00 = fx/z, J02 = -fx tx/z^2, J11 = fy/z, J12 = -fy ty/z^2.
  float gJ00 = 0.f, gJ02 = 0.f, gJ11 = 0.f, gJ12 = 0.f;
#pragma unroll
  for (int c = 0; c < 3; ++c) {
    gJ00 += dA0[c] * cam.view[4 * c + 0];
    gJ02 += dA0[c] * cam.view[4 * c + 2];
    gJ11 += dA1[c] * cam.view[4 * c + 1];
    gJ12 += dA1[c] * cam.view[4 * c + 2];
  }
  const float iz = 1.f / J.tz, iz2 = iz * iz, iz3 = iz2 * iz;
  const float dJ02_dtx = -cam.fx * iz2, dJ12_dty = -cam.fy * iz2;
  const float dJ00_dz = -cam.fx * iz2, dJ11_dz = -cam.fy * iz2;
  const float dJ02_dz = 2.f * cam.fx * J.tx * iz3, dJ12_dz = 2.f * cam.fy * J.ty * iz3;
  float dt[3];
  dt[0] = J.clamp_x ? 0.f : gJ02 * dJ02_dtx;
  dt[1] = J.clamp_y ? 0.f : gJ12 * dJ12_dty;
  dt[2] = gJ00 * dJ00_dz + gJ11 * dJ11_dz + gJ02 * dJ02_dz + gJ12 * dJ12_dz;
  if (o.dinvdepth) dt[2] -= o.dinvdepth[i] * iz2;  // d(1/z)/dz = -1/z^2
  // t = W p + b: dL/dp = W^T dL/dt.
  float dm[3];
#pragma unroll
  for (int k = 0; k < 3; ++k)
    dm[k] = cam.view[4 * k + 0] * dt[0] + cam.view[4 * k + 1] * dt[1] +
            cam.view[4 * k + 2] * dt[2];
  // Screen mean in NDC, h.xy / (h.w + 1e-7) with h = proj [p, 1]:
  // d ndc / dp_k = (proj_row(k) - ndc * proj_w(k)) / (h.w + 1e-7).
  {
    const float iw = 1.f / (affine_w(cam.proj, p) + 0.0000001f);
    const Vec3 h = affine3(cam.proj, p);
    const float nx = h.x * iw, ny = h.y * iw;
    const float gx = o.dmean2d[3 * i], gy = o.dmean2d[3 * i + 1];
#pragma unroll
    for (int k = 0; k < 3; ++k) {
      const float pw = cam.proj[4 * k + 3];
      dm[k] += iw * ((cam.proj[4 * k + 0] - nx * pw) * gx + (cam.proj[4 * k + 1] - ny * pw) * gy);
    }
  }
  // (The SH colour's share of dmeans, the view direction's adjoint, is added
  // by sh_backward_kernel afterwards.)
#pragma unroll
  for (int k = 0; k < 3; ++k) o.dmeans[3 * i + k] += dm[k];
  if (cov3d_precomp) return;
  // S3 = M M^T with M = R diag(s): dL/dM = 2 G3 M; M_rc = R_rc s_c.
  const float s[3] = {scale_modifier * scales[3 * i], scale_modifier * scales[3 * i + 1],
                      scale_modifier * scales[3 * i + 2]};
  const float q[4] = {rotations[4 * i], rotations[4 * i + 1], rotations[4 * i + 2],
                      rotations[4 * i + 3]};
  float R[9];
  rotation(q, R);
  float dR[9];
#pragma unroll
  for (int c = 0; c < 3; ++c) {
    float ds = 0.f;
#pragma unroll
    for (int r = 0; r < 3; ++r) {
      const float dM = 2.f * (G3[3 * r] * R[c] * s[c] + G3[3 * r + 1] * R[3 + c] * s[c] +
                              G3[3 * r + 2] * R[6 + c] * s[c]);
      ds += dM * R[3 * r + c];
      dR[3 * r + c] = dM * s[c];
    }
    o.dscales[3 * i + c] = scale_modifier * ds;
  }
  float dq4[4];
  rotation_vjp(q, dR, dq4);
#pragma unroll
  for (int k = 0; k < 4; ++k) o.drotations[4 * i + k] = dq4[k];
}

// SH colour of every drawn Gaussian: sh_backward.cu (one translation unit
// without multiply-add contraction with the data-parallel colour production).
cudaError_t launch_sh_colour(int P, int degree, const float* means, ShSource sh,
                             const float* campos, const int* radii, bool* clamped, float* rgb,
                             cudaStream_t stream);


// The SH backward (sh_backward.cu, compiled without contraction so that the
// data-parallel exchange's seed form rounds exactly alike).
cudaError_t launch_sh_backward(int P, int degree, const float* means, ShSource sh,
                               const float* campos, const bool* clamped, const int* radii,
                               const float* dcolor, float* dsh, float* dmeans,
                               cudaStream_t stream);

}  // namespace raster
}  // namespace clad3dgs

// ===========================================================================
// C ABI.

using namespace clad3dgs;
using namespace clad3dgs::raster;

namespace {

int status_of(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return CLAD3DGS_OK;
  cudaGetLastError();
  return fail(CLAD3DGS_CUDA_ERROR, std::string(what) + ": " + cudaGetErrorString(e));
}

int bits_for(uint32_t v) {
  int b = 0;
  while (b < 32 && (v >> b) != 0) ++b;
  return b;
}

// Depth order, row counts and their scan; reads the totals (tile instances,
// row pairs) back to the host. Needs g.depth, g.tiles, g.rows.
int order_and_count(int P, GeomState& g, uint32_t& instances, uint32_t& pairs,
                    cudaStream_t stream) {
  const int blocks = (P + 255) / 256;
  depth_key_kernel<<<blocks, 256, 0, stream>>>(P, g);
  cudaError_t e = cub::DeviceRadixSort::SortPairs(g.order_tmp, g.order_bytes, g.depth_keys,
                                                  g.depth_sorted, g.ids, g.order, P, 0, 32,
                                                  stream);
  if (e != cudaSuccess) return status_of(e, "depth order");
  gather_rows_kernel<<<blocks, 256, 0, stream>>>(P, g);
  e = cub::DeviceScan::InclusiveSum(g.scan_tmp, g.scan_bytes, g.depth_keys, g.offsets, P,
                                    stream);
  if (e != cudaSuccess) return status_of(e, "row scan");
  e = cub::DeviceReduce::Sum(g.scan_tmp, g.scan_bytes, g.tiles, g.totals, P, stream);
  if (e != cudaSuccess) return status_of(e, "instance count");
  e = cudaMemcpyAsync(g.totals + 1, g.offsets + P - 1, sizeof(uint32_t),
                      cudaMemcpyDeviceToDevice, stream);
  uint32_t host[2] = {0, 0};
  if (e == cudaSuccess)
    e = cudaMemcpyAsync(host, g.totals, sizeof(host), cudaMemcpyDeviceToHost, stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(stream);
  if (e != cudaSuccess) return status_of(e, "reading the instance count");
  instances = host[0];
  pairs = host[1];
  return CLAD3DGS_OK;
}

// Per-tile lists and ranges from the depth order (see "Binning" above).
int bin_instances(int P, const GeomState& g, int grid_x, int grid_y, uint32_t n, uint32_t m,
                  const BinningState& b, const ImageState& img, cudaStream_t stream) {
  if (grid_x > 0xffff) return fail(CLAD3DGS_INVALID_ARGUMENT, "image too wide for binning");
  const int tiles = grid_x * grid_y;
  const size_t place_bytes = place_shared_bytes(grid_x);
  {
    int device = 0, limit = 0;
    cudaError_t e = cudaGetDevice(&device);
    if (e == cudaSuccess)
      e = cudaDeviceGetAttribute(&limit, cudaDevAttrMaxSharedMemoryPerBlockOptin, device);
    if (e != cudaSuccess) return status_of(e, "device attributes");
    if (place_bytes + 1024 > size_t(limit))
      return fail(CLAD3DGS_INVALID_ARGUMENT, "image too wide for binning");
    if (place_bytes > 48 * 1024) {
      e = cudaFuncSetAttribute(place_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               int(place_bytes));
      if (e != cudaSuccess) return status_of(e, "placement shared memory");
    }
  }
  constexpr int kEmitThreads = 32 * kEmitWarps;
  emit_rows_kernel<<<(P + kEmitThreads - 1) / kEmitThreads, kEmitThreads, 0, stream>>>(
      P, g, grid_x, grid_y, b.pair_rows, b.pair_spans);
  size_t sort_bytes = b.sort_bytes;
  cudaError_t e = cub::DeviceRadixSort::SortPairs(
      b.sort_tmp, sort_bytes, b.pair_rows, b.pair_rows_sorted, b.pair_spans,
      b.pair_spans_sorted, int(m), 0, bits_for(uint32_t(grid_y)), stream);
  if (e != cudaSuccess) return status_of(e, "row sort");
  row_layout_kernel<<<1, 1024, 0, stream>>>(m, grid_y, b.pair_rows_sorted, b.row_start,
                                            b.chunk_first);
  tile_count_kernel<<<b.max_chunks, kBinThreads, (grid_x + 1) * sizeof(int), stream>>>(
      grid_x, grid_y, b.pair_spans_sorted, b.row_start, b.chunk_first, b.chunk_counts);
  tile_totals_kernel<<<dim3((grid_x + 31) / 32, grid_y), kBinThreads, 0, stream>>>(
      grid_x, b.chunk_first, b.chunk_counts, b.tile_total);
  size_t scan_bytes = b.scan_bytes;
  e = cub::DeviceScan::ExclusiveSum(b.scan_tmp, scan_bytes, b.tile_total, b.tile_start, tiles,
                                    stream);
  if (e != cudaSuccess) return status_of(e, "tile scan");
  tile_ranges_kernel<<<(tiles + 255) / 256, 256, 0, stream>>>(tiles, b.tile_start,
                                                              b.tile_total, img.ranges);
  place_kernel<<<b.max_chunks, kBinThreads, place_bytes, stream>>>(
      grid_x, grid_y, n, b.pair_spans_sorted, b.row_start, b.chunk_first, b.chunk_counts,
      b.tile_start, b.values);
  return status_of(cudaPeekAtLastError(), "binning");
}

Camera make_camera(const float* view, const float* proj, const float* campos, int width,
                   int height, float tan_x, float tan_y) {
  Camera c;
  c.view = view;
  c.proj = proj;
  c.campos = campos;
  c.tan_x = tan_x;
  c.tan_y = tan_y;
  c.fx = width / (2.f * tan_x);
  c.fy = height / (2.f * tan_y);
  c.width = width;
  c.height = height;
  c.grid_x = (width + kTileX - 1) / kTileX;
  c.grid_y = (height + kTileY - 1) / kTileY;
  return c;
}

}  // namespace

extern "C" size_t clad3dgs_raster_geom_bytes(int P) { return P > 0 ? geom_bytes(P) : 0; }
extern "C" size_t clad3dgs_raster_image_bytes(int width, int height) {
  const int tiles = ((width + kTileX - 1) / kTileX) * ((height + kTileY - 1) / kTileY);
  return image_bytes(width * height, tiles);
}
extern "C" size_t clad3dgs_raster_binning_bytes(int instances, int row_pairs, int width,
                                                int height) {
  if (instances <= 0 || row_pairs <= 0 || width <= 0 || height <= 0) return 0;
  return binning_bytes(uint32_t(instances), uint32_t(row_pairs), (width + kTileX - 1) / kTileX,
                       (height + kTileY - 1) / kTileY);
}

// Forward. The view-space / projection matrices, campos and bg are device
// pointers; the three buffers are requested from the caller through `alloc`
// (geom first, then image, then binning once the number of tile instances is
// known), as the renderer's resizable buffers are.
extern "C" int clad3dgs_raster_forward(
    int P, int degree, const float* bg, const float* means, const float* colors_precomp,
    const float* opacities, const float* scales, float scale_modifier,
    const float* rotations, const float* cov3d_precomp, const float* view,
    const float* proj, float tan_x, float tan_y, int height, int width,
    const float* sh_packed, const float* sh_dc, const float* sh_rest, const float* campos,
    int antialiasing, clad3dgs_alloc_fn alloc, void* alloc_ctx, float* out_color,
    float* out_invdepth, int* radii, int* num_rendered, cudaStream_t stream) {
  *num_rendered = 0;
  if (degree < 0 || degree > 3)
    return fail(CLAD3DGS_INVALID_ARGUMENT, "SH degree must be between zero and three");
  if (width <= 0 || height <= 0)
    return fail(CLAD3DGS_INVALID_ARGUMENT, "image size must be positive");
  if (P > 0 && !colors_precomp && !(sh_packed || (sh_dc && sh_rest)))
    return fail(CLAD3DGS_INVALID_ARGUMENT, "forward: neither colours nor SH coefficients");
  const Camera cam = make_camera(view, proj, campos, width, height, tan_x, tan_y);
  const int tiles = cam.grid_x * cam.grid_y;
  char* image_base = alloc(alloc_ctx, 1, image_bytes(width * height, tiles));
  if (!image_base) return fail(CLAD3DGS_INVALID_ARGUMENT, "image buffer allocation failed");
  ImageState img = image_from(image_base, width * height, tiles);
  cudaError_t e = cudaMemsetAsync(img.ranges, 0, sizeof(uint2) * tiles, stream);
  if (e != cudaSuccess) return status_of(e, "clearing tile ranges");
  if (P > 0) {
    char* geom_base = alloc(alloc_ctx, 0, geom_bytes(P));
    if (!geom_base) return fail(CLAD3DGS_INVALID_ARGUMENT, "geometry buffer allocation failed");
    GeomState g = geom_from(geom_base, P);
    const ShSource sh{sh_packed, sh_dc, sh_rest};
    preprocess_kernel<<<(P + 255) / 256, 256, 0, stream>>>(
        P, means, scales, scale_modifier, rotations, opacities, colors_precomp, cov3d_precomp,
        cam, antialiasing != 0, g, radii);
    if (!colors_precomp) {
      e = launch_sh_colour(P, degree, means, sh, campos, g.radii, g.clamped, g.rgb, stream);
      if (e != cudaSuccess) return status_of(e, "SH colour");
    }
    uint32_t total = 0, pairs = 0;
    int status = order_and_count(P, g, total, pairs, stream);
    if (status != CLAD3DGS_OK) return status;
    if (total > uint32_t(INT32_MAX) || pairs > uint32_t(INT32_MAX))
      return fail(CLAD3DGS_INVALID_ARGUMENT, "more than 2^31 - 1 tile instances");
    *num_rendered = int(total);
    if (total > 0) {
      char* bin_base =
          alloc(alloc_ctx, 2, binning_bytes(total, pairs, cam.grid_x, cam.grid_y));
      if (!bin_base) return fail(CLAD3DGS_INVALID_ARGUMENT, "binning buffer allocation failed");
      BinningState b = binning_from(bin_base, total, pairs, cam.grid_x, cam.grid_y);
      status = bin_instances(P, g, cam.grid_x, cam.grid_y, total, pairs, b, img, stream);
      if (status != CLAD3DGS_OK) return status;
      render_forward_kernel<<<dim3(cam.grid_x, cam.grid_y), kTilePixels, 0, stream>>>(
          img.ranges, b.values, width, height, cam.grid_x, g.mean2d, g.rgb,
          g.conic_opacity, g.depth, bg, img.final_t, img.n_contrib, out_color, out_invdepth);
      return status_of(cudaPeekAtLastError(), "forward kernels");
    }
  }
  // Nothing to draw: background everywhere.
  render_forward_kernel<<<dim3(cam.grid_x, cam.grid_y), kTilePixels, 0, stream>>>(
      img.ranges, nullptr, width, height, cam.grid_x, nullptr, nullptr, nullptr, nullptr, bg,
      img.final_t, img.n_contrib, out_color, out_invdepth);
  return status_of(cudaPeekAtLastError(), "forward kernels");
}

// Pixel backward only (used by the 2D benchmark and tests). dmean2d [P][3],
// dconic [P][4], dopacity [P], dcolor [P][3], dinvdepth [P] (nullable) are
// accumulated into (callers zero them).
extern "C" int clad3dgs_raster_render_backward(
    int P, int width, int height, const float* bg, const void* geom_buffer,
    const void* binning_buffer, int num_rendered, const void* image_buffer,
    const float* dpixels, const float* dinvdepth_pixels, float* dmean2d, float* dconic,
    float* dopacity, float* dcolor, float* dinvdepth, int mode, cudaStream_t stream) {
  if (mode < 0 || mode > 2)
    return fail(CLAD3DGS_INVALID_ARGUMENT, "accumulation mode must be 0, 1 or 2");
  if (P <= 0 || num_rendered <= 0) return CLAD3DGS_OK;
  const int gx = (width + kTileX - 1) / kTileX, gy = (height + kTileY - 1) / kTileY;
  GeomState g = geom_from(static_cast<char*>(const_cast<void*>(geom_buffer)), P);
  ImageState img = image_from(static_cast<char*>(const_cast<void*>(image_buffer)),
                              width * height, gx * gy);
  const uint32_t* point_list = point_list_from(binning_buffer);
  PixelGrads o{dmean2d, dconic, dopacity, dcolor, dinvdepth};
  const dim3 grid(gx, gy);
  if (mode == 0)
    render_backward_kernel<0><<<grid, kTilePixels, 0, stream>>>(
        img.ranges, point_list, width, height, gx, bg, g.mean2d, g.conic_opacity, g.rgb,
        g.depth, img.final_t, img.n_contrib, dpixels, dinvdepth_pixels, o);
  else if (mode == 1)
    render_backward_kernel<1><<<grid, kTilePixels, 0, stream>>>(
        img.ranges, point_list, width, height, gx, bg, g.mean2d, g.conic_opacity, g.rgb,
        g.depth, img.final_t, img.n_contrib, dpixels, dinvdepth_pixels, o);
  else
    render_backward_pairs_kernel<<<grid, kPairThreads, 0, stream>>>(
        img.ranges, point_list, width, height, gx, bg, g.mean2d, g.conic_opacity, g.rgb,
        g.depth, img.final_t, img.n_contrib, dpixels, dinvdepth_pixels, o);
  return status_of(cudaPeekAtLastError(), "pixel backward");
}

extern "C" int clad3dgs_raster_count_accumulation(int P, int width, int height,
                                                  const void* geom_buffer,
                                                  const void* binning_buffer,
                                                  int num_rendered, const void* image_buffer,
                                                  unsigned long long* counts,
                                                  cudaStream_t stream) {
  if (!counts) return fail(CLAD3DGS_INVALID_ARGUMENT, "count pass: null counts");
  cudaError_t e = cudaMemsetAsync(counts, 0, 3 * sizeof(unsigned long long), stream);
  if (e != cudaSuccess) return status_of(e, "count pass");
  if (P <= 0 || num_rendered <= 0) return CLAD3DGS_OK;
  if (!geom_buffer || !binning_buffer || !image_buffer)
    return fail(CLAD3DGS_INVALID_ARGUMENT, "count pass: null buffer");
  const int gx = (width + kTileX - 1) / kTileX, gy = (height + kTileY - 1) / kTileY;
  GeomState g = geom_from(static_cast<char*>(const_cast<void*>(geom_buffer)), P);
  ImageState img = image_from(static_cast<char*>(const_cast<void*>(image_buffer)),
                              width * height, gx * gy);
  count_accumulation_kernel<<<dim3(gx, gy), kTilePixels, 0, stream>>>(
      img.ranges, point_list_from(binning_buffer), width, height, gx, g.mean2d,
      g.conic_opacity, img.n_contrib, counts);
  return status_of(cudaPeekAtLastError(), "count pass");
}

extern "C" int clad3dgs_warp_accumulate_probe(int mode, int n, int fields, const int* keys,
                                              const unsigned char* active,
                                              const float* values, float* out, int rows,
                                              int* grouped, int block_x, int block_y,
                                              int block_z, cudaStream_t stream) {
  if (mode < 0 || mode > 2)
    return fail(CLAD3DGS_INVALID_ARGUMENT, "accumulation mode must be 0, 1 or 2");
  if (fields < 1 || fields > 16)
    return fail(CLAD3DGS_INVALID_ARGUMENT, "between 1 and 16 fields per lane");
  const long block = long(block_x) * block_y * block_z;
  if (block_x < 1 || block_y < 1 || block_z < 1 || block % 32 != 0 || block > 1024)
    return fail(CLAD3DGS_INVALID_ARGUMENT, "blocks must hold whole warps (at most 1024 threads)");
  if (n < 0 || rows < 0) return fail(CLAD3DGS_INVALID_ARGUMENT, "negative size");
  if (n == 0) return CLAD3DGS_OK;
  if (!keys || !active || !values || !out || !grouped)
    return fail(CLAD3DGS_INVALID_ARGUMENT, "warp probe: null pointer");
  const unsigned grid = unsigned((long(n) + block - 1) / block);
  warp_probe_kernel<<<grid, dim3(block_x, block_y, block_z), 0, stream>>>(
      mode, n, fields, keys, active, values, out, rows, grouped);
  return status_of(cudaPeekAtLastError(), "warp probe");
}

// Full backward. Outputs (zeroed by the caller): dmean2d [P][3], dcolor [P][3],
// dopacity [P], dmeans [P][3], dcov3d [P][6], dsh [P][16][3] (null when
// consume_sh), dscales [P][3], drotations [P][4]. With consume_sh, the SH
// adjoint is not written: dcolor (masked by the clamp flags) feeds the fused
// SH + Adam kernel, which updates dc/rest and both moments in place and adds
// the direction adjoint into dmeans (sh_consumer_split_torch_adam semantics).
extern "C" int clad3dgs_raster_backward(
    int P, int degree, const float* bg, const float* means, const int* radii,
    const float* colors_precomp, const float* opacities, const float* scales,
    float scale_modifier, const float* rotations, const float* cov3d_precomp,
    const float* view, const float* proj, float tan_x, float tan_y, int height, int width,
    const float* dpixels, const float* dinvdepth_pixels, const float* sh_packed,
    const float* sh_dc, const float* sh_rest, const float* campos, const void* geom_buffer,
    int num_rendered, const void* binning_buffer, const void* image_buffer,
    int antialiasing, float* dmean2d, float* dcolor, float* dopacity, float* dmeans,
    float* dcov3d, float* dsh, float* dscales, float* drotations, float* dconic_scratch,
    float* dinvdepth_scratch, int mode, int consume_sh, float* dc, float* rest,
    float* dc_first, float* dc_second, float* rest_first, float* rest_second,
    TorchAdamConfig config, float* xyz_first, float* xyz_second, double xyz_rate,
    TorchAdamConfig xyz_config, cudaStream_t stream) {
  if (degree < 0 || degree > 3)
    return fail(CLAD3DGS_INVALID_ARGUMENT, "SH degree must be between zero and three");
  if (consume_sh < 0 || consume_sh > 2)
    return fail(CLAD3DGS_INVALID_ARGUMENT, "consume_sh must be 0, 1 or 2");
  if (P <= 0) return CLAD3DGS_OK;
  if (!colors_precomp && consume_sh != 2 && !(sh_packed || (sh_dc && sh_rest)))
    return fail(CLAD3DGS_INVALID_ARGUMENT, "backward: neither colours nor SH coefficients");
  int status = clad3dgs_raster_render_backward(
      P, width, height, bg, geom_buffer, binning_buffer, num_rendered, image_buffer, dpixels,
      dinvdepth_pixels, dmean2d, dconic_scratch, dopacity, dcolor,
      dinvdepth_pixels ? dinvdepth_scratch : nullptr, mode, stream);
  if (status != CLAD3DGS_OK) return status;
  const Camera cam = make_camera(view, proj, campos, width, height, tan_x, tan_y);
  GeomState g = geom_from(static_cast<char*>(const_cast<void*>(geom_buffer)), P);
  const ShSource sh{sh_packed, sh_dc, sh_rest};
  GeomGrads o{dmean2d, dconic_scratch, dopacity, dinvdepth_pixels ? dinvdepth_scratch : nullptr,
              dmeans, dcov3d, dscales, drotations};
  const bool from_sh = colors_precomp == nullptr && !consume_sh;
  preprocess_backward_kernel<<<(P + 255) / 256, 256, 0, stream>>>(
      P, means, scales, scale_modifier, rotations, opacities, cov3d_precomp, cam,
      antialiasing != 0, radii, g, o);
  if (from_sh) {
    const cudaError_t e = launch_sh_backward(P, degree, means, sh, campos, g.clamped, radii,
                                             dcolor, dsh, dmeans, stream);
    if (e != cudaSuccess) return status_of(e, "SH backward");
  }
  cudaError_t e = cudaPeekAtLastError();
  if (e != cudaSuccess) return status_of(e, "geometry backward");
  if (consume_sh == 1 && colors_precomp == nullptr) {
    if (xyz_first)  // the positions' Adam too; means are updated after every read of them
      return clad3dgs_sh_consume_xyz(P, degree, const_cast<float*>(means), radii, sh_packed,
                                     g.clamped, campos, dcolor, dmeans, dc, rest, dc_first,
                                     dc_second, rest_first, rest_second, config, xyz_first,
                                     xyz_second, xyz_rate, xyz_config, stream);
    return clad3dgs_sh_consume_split_torch_adam(
        P, degree, means, radii, sh_packed, g.clamped, campos, dcolor, dmeans, dc, rest,
        dc_first, dc_second, rest_first, rest_second, config, stream);
  }
  return CLAD3DGS_OK;
}

namespace clad3dgs {
namespace raster {
__global__ void sh_seed_kernel(int P, const int* __restrict__ radii,
                               const bool* __restrict__ clamped,
                               const float* __restrict__ dcolor, float4* __restrict__ seeds) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= P) return;
  float4 s = make_float4(0.f, 0.f, 0.f, 0.f);
  if (radii[i] > 0) {
    s.x = clamped[3 * i] ? 0.f : dcolor[3 * i];
    s.y = clamped[3 * i + 1] ? 0.f : dcolor[3 * i + 1];
    s.z = clamped[3 * i + 2] ? 0.f : dcolor[3 * i + 2];
    s.w = 1.f;
  }
  seeds[i] = s;
}
}  // namespace raster
}  // namespace clad3dgs

extern "C" int clad3dgs_raster_sh_backward(int P, int degree, const float* means,
                                           const int* radii, const float* sh_packed,
                                           const float* sh_dc, const float* sh_rest,
                                           const float* campos, const bool* clamped,
                                           const float* dcolor, float* dsh, float* dmeans,
                                           cudaStream_t stream) {
  if (degree < 0 || degree > 3)
    return fail(CLAD3DGS_INVALID_ARGUMENT, "SH degree must be between zero and three");
  if (P <= 0) return CLAD3DGS_OK;
  if (!means || !radii || !campos || !clamped || !dcolor || !dmeans ||
      !(sh_packed || (sh_dc && sh_rest)))
    return fail(CLAD3DGS_INVALID_ARGUMENT, "SH backward: null pointer");
  return status_of(launch_sh_backward(P, degree, means, ShSource{sh_packed, sh_dc, sh_rest},
                                      campos, clamped, radii, dcolor, dsh, dmeans, stream),
                   "SH backward");
}

extern "C" int clad3dgs_raster_sh_seeds(int P, const int* radii, const void* geom_buffer,
                                        const float* dcolor, float* seeds,
                                        cudaStream_t stream) {
  if (P <= 0) return CLAD3DGS_OK;
  if (!radii || !geom_buffer || !dcolor || !seeds)
    return fail(CLAD3DGS_INVALID_ARGUMENT, "SH seeds: null pointer");
  if (reinterpret_cast<uintptr_t>(seeds) & 15u)
    return fail(CLAD3DGS_INVALID_ARGUMENT, "SH seeds: the seed array must be 16-byte aligned");
  const GeomState g = geom_from(static_cast<char*>(const_cast<void*>(geom_buffer)), P);
  sh_seed_kernel<<<(P + 255) / 256, 256, 0, stream>>>(P, radii, g.clamped, dcolor,
                                                      reinterpret_cast<float4*>(seeds));
  return status_of(cudaPeekAtLastError(), "SH seeds");
}

namespace clad3dgs {
namespace raster {
__global__ void fill_2d_kernel(int P, const float* __restrict__ mean2d,
                               const float* __restrict__ conic_opacity,
                               const float* __restrict__ rgb, const float* __restrict__ depth,
                               const int* __restrict__ radii, int grid_x, int grid_y,
                               GeomState g) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= P) return;
  const float px = mean2d[2 * i], py = mean2d[2 * i + 1];
  const int r = radii[i];
  g.mean2d[i] = make_float2(px, py);
  g.conic_opacity[i] = make_float4(conic_opacity[4 * i], conic_opacity[4 * i + 1],
                                   conic_opacity[4 * i + 2], conic_opacity[4 * i + 3]);
  g.rgb[3 * i] = rgb[3 * i];
  g.rgb[3 * i + 1] = rgb[3 * i + 1];
  g.rgb[3 * i + 2] = rgb[3 * i + 2];
  g.depth[i] = depth[i];
  g.radii[i] = r;
  const Footprint f = make_footprint(px, py, g.conic_opacity[i], r, grid_x, grid_y);
  const uint32_t n = r > 0 ? footprint_tiles(f) : 0u;
  g.tiles[i] = n;
  g.rows[i] = n ? uint32_t(f.y1 - f.y0) : 0u;
}
}  // namespace raster
}  // namespace clad3dgs

// Binning + forward compositing of already projected 2D Gaussians (the pixel
// stage alone, for the 2D benchmark configuration). Inputs: mean2d [P][2]
// pixels, conic_opacity [P][4], rgb [P][3], depth [P], radii [P]. The geom
// buffer is filled from them so clad3dgs_raster_render_backward can follow.
extern "C" int clad3dgs_raster_forward_2d(int P, const float* mean2d,
                                          const float* conic_opacity, const float* rgb,
                                          const float* depth, const int* radii, int width,
                                          int height, const float* bg,
                                          clad3dgs_alloc_fn alloc, void* alloc_ctx,
                                          float* out_color, float* out_invdepth,
                                          int* num_rendered, cudaStream_t stream) {
  *num_rendered = 0;
  if (P <= 0 || width <= 0 || height <= 0)
    return fail(CLAD3DGS_INVALID_ARGUMENT, "need Gaussians and a positive image size");
  const int gx = (width + kTileX - 1) / kTileX, gy = (height + kTileY - 1) / kTileY;
  char* image_base = alloc(alloc_ctx, 1, image_bytes(width * height, gx * gy));
  char* geom_base = alloc(alloc_ctx, 0, geom_bytes(P));
  if (!image_base || !geom_base)
    return fail(CLAD3DGS_INVALID_ARGUMENT, "buffer allocation failed");
  ImageState img = image_from(image_base, width * height, gx * gy);
  GeomState g = geom_from(geom_base, P);
  cudaError_t e = cudaMemsetAsync(img.ranges, 0, sizeof(uint2) * gx * gy, stream);
  if (e != cudaSuccess) return status_of(e, "clearing tile ranges");
  fill_2d_kernel<<<(P + 255) / 256, 256, 0, stream>>>(P, mean2d, conic_opacity, rgb, depth,
                                                      radii, gx, gy, g);
  uint32_t total = 0, pairs = 0;
  int status = order_and_count(P, g, total, pairs, stream);
  if (status != CLAD3DGS_OK) return status;
  if (total > uint32_t(INT32_MAX) || pairs > uint32_t(INT32_MAX))
    return fail(CLAD3DGS_INVALID_ARGUMENT, "more than 2^31 - 1 tile instances");
  *num_rendered = int(total);
  if (total == 0) return CLAD3DGS_OK;
  char* bin_base = alloc(alloc_ctx, 2, binning_bytes(total, pairs, gx, gy));
  if (!bin_base) return fail(CLAD3DGS_INVALID_ARGUMENT, "binning buffer allocation failed");
  BinningState b = binning_from(bin_base, total, pairs, gx, gy);
  status = bin_instances(P, g, gx, gy, total, pairs, b, img, stream);
  if (status != CLAD3DGS_OK) return status;
  render_forward_kernel<<<dim3(gx, gy), kTilePixels, 0, stream>>>(
      img.ranges, b.values, width, height, gx, g.mean2d, g.rgb, g.conic_opacity, g.depth, bg,
      img.final_t, img.n_contrib, out_color, out_invdepth);
  return status_of(cudaPeekAtLastError(), "forward kernels");
}
