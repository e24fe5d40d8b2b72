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
  if (colors_precomp) {
#pragma unroll
    for (int k = 0; k < 3; ++k) g.rgb[3 * i + k] = colors_precomp[3 * i + k];
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
      const float power = -0.5f * (co.x * dx * dx + co.z * dy * dy) - co.y * dx * dy;
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
// Pixel backward.

struct PixelGrads {
  float* dmean2d;    // [P][3]
  float* dconic;     // [P][4] (a, b, -, c)
  float* dopacity;   // [P]
  float* dcolor;     // [P][3]
  float* dinvdepth;  // [P] or null
};

// Address of adjoint field f (0-2 RGB, 3-4 mean x/y, 5-7 conic a/b/c,
// 8 opacity, 9 inverse depth) of Gaussian id.
__device__ __forceinline__ float* field_address(const PixelGrads& o, uint32_t id, int f) {
  switch (f) {
    case 0: case 1: case 2: return o.dcolor + 3 * size_t(id) + f;
    case 3: case 4: return o.dmean2d + 3 * size_t(id) + (f - 3);
    case 5: return o.dconic + 4 * size_t(id);
    case 6: return o.dconic + 4 * size_t(id) + 1;
    case 7: return o.dconic + 4 * size_t(id) + 3;
    case 8: return o.dopacity + id;
    default: return o.dinvdepth + id;
  }
}

// Sums v[0..9] over the warp; afterwards lane L holds the total of field
// (L >> 1) & 15 (lanes L and L ^ 1 hold the same value). Each butterfly step
// halves the number of fields a lane keeps, so 16 shuffles cover 10 fields.
__device__ __forceinline__ float transpose_reduce(float v[16], int lane) {
#pragma unroll
  for (int step = 0; step < 4; ++step) {
    const int half = 8 >> step;          // fields kept after this step
    const int mask = 16 >> step;         // lane bit that picks the half
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
  const bool inside = px < width && py < height;
  const int pix = py * width + px;
  const int lane = threadIdx.x & 31;
  const float fx = (float)px, fy = (float)py;
  const uint2 range = ranges[tile];
  __shared__ uint32_t s_id[kBatch];
  __shared__ uint32_t s_last_max;
  __shared__ float2 s_xy[kBatch];
  __shared__ float4 s_co[kBatch];
  __shared__ float s_rgb[3 * kBatch];
  __shared__ float s_inv[kBatch];
  const int hw = width * height;
  const float T_final = inside ? final_t[pix] : 0.f;
  float T = T_final;
  const uint32_t last = inside ? n_contrib[pix] : 0;
  // No pixel of the tile has a contributor past the largest last-contributor
  // index, so the back-to-front walk starts there instead of at the end of the
  // tile's range (identical results; the skipped Gaussians contribute nothing).
  if (threadIdx.x == 0) s_last_max = 0;
  __syncthreads();
  const uint32_t warp_max = __reduce_max_sync(0xffffffffu, last);
  if (lane == 0) atomicMax(&s_last_max, warp_max);
  __syncthreads();
  const int todo = int(s_last_max);
  uint32_t contributor = todo;
  float dpix[3] = {0.f, 0.f, 0.f}, dinv = 0.f;
  if (inside) {
    dpix[0] = dpixels[pix];
    dpix[1] = dpixels[hw + pix];
    dpix[2] = dpixels[2 * hw + pix];
    if (dinvdepth_pixels) dinv = dinvdepth_pixels[pix];
  }
  const float bg_dot = bg[0] * dpix[0] + bg[1] * dpix[1] + bg[2] * dpix[2];
  float acc[3] = {0.f, 0.f, 0.f}, acc_inv = 0.f;
  float last_alpha = 0.f, last_rgb[3] = {0.f, 0.f, 0.f}, last_inv = 0.f;
  const float ddx = 0.5f * width, ddy = 0.5f * height;
  for (int base = 0; base < todo; base += kBatch) {
    __syncthreads();
    const int k = base + threadIdx.x;
    if (k < todo) {
      const uint32_t id = point_list[range.x + todo - k - 1];
      s_id[threadIdx.x] = id;
      s_xy[threadIdx.x] = mean2d[id];
      s_co[threadIdx.x] = conic_opacity[id];
      s_rgb[3 * threadIdx.x] = rgb[3 * id];
      s_rgb[3 * threadIdx.x + 1] = rgb[3 * id + 1];
      s_rgb[3 * threadIdx.x + 2] = rgb[3 * id + 2];
      s_inv[threadIdx.x] = 1.f / depth[id];
    }
    __syncthreads();
    const int count = min(kBatch, todo - base);
    for (int j = 0; j < count; ++j) {
      --contributor;
      bool contrib = inside && contributor < last;
      const float4 co = s_co[j];
      const float dx = s_xy[j].x - fx, dy = s_xy[j].y - fy;
      const float power = -0.5f * (co.x * dx * dx + co.z * dy * dy) - co.y * dx * dy;
      contrib = contrib && power <= 0.f;
      const float G = __expf(power);
      const float alpha = fminf(kMaxAlpha, co.w * G);
      contrib = contrib && alpha >= kMinAlpha;
      float f[16];
      if (!contrib) continue;
      {
        const float inv_keep = 1.f / (1.f - alpha);  // one reciprocal for T and the bg term
        T = T * inv_keep;
        const float w = alpha * T;
        float dl_dalpha = 0.f;
#pragma unroll
        for (int ch = 0; ch < 3; ++ch) {
          const float cc = s_rgb[3 * j + ch];
          acc[ch] = last_alpha * last_rgb[ch] + (1.f - last_alpha) * acc[ch];
          last_rgb[ch] = cc;
          dl_dalpha += (cc - acc[ch]) * dpix[ch];
          f[ch] = w * dpix[ch];
        }
        const float inv = s_inv[j];
        acc_inv = last_alpha * last_inv + (1.f - last_alpha) * acc_inv;
        last_inv = inv;
        dl_dalpha += (inv - acc_inv) * dinv;
        f[9] = w * dinv;
        dl_dalpha *= T;
        last_alpha = alpha;
        dl_dalpha += (-T_final * inv_keep) * bg_dot;
        const float dl_dg = co.w * dl_dalpha;
        const float gdx = G * dx, gdy = G * dy;
        const float dg_ddx = -gdx * co.x - gdy * co.y;
        const float dg_ddy = -gdy * co.z - gdx * co.y;
        f[3] = dl_dg * dg_ddx * ddx;
        f[4] = dl_dg * dg_ddy * ddy;
        f[5] = -0.5f * gdx * dx * dl_dg;
        f[6] = -0.5f * gdx * dy * dl_dg;
        f[7] = -0.5f * gdy * dy * dl_dg;
        f[8] = G * dl_dalpha;
      }
      const uint32_t id = s_id[j];
      const int nf = out.dinvdepth ? 10 : 9;
      if constexpr (Mode == 0) {
        atomicAdd(out.dcolor + 3 * size_t(id), f[0]);
        atomicAdd(out.dcolor + 3 * size_t(id) + 1, f[1]);
        atomicAdd(out.dcolor + 3 * size_t(id) + 2, f[2]);
        atomicAdd(out.dmean2d + 3 * size_t(id), f[3]);
        atomicAdd(out.dmean2d + 3 * size_t(id) + 1, f[4]);
        atomicAdd(out.dconic + 4 * size_t(id), f[5]);
        atomicAdd(out.dconic + 4 * size_t(id) + 1, f[6]);
        atomicAdd(out.dconic + 4 * size_t(id) + 3, f[7]);
        atomicAdd(out.dopacity + id, f[8]);
        if (out.dinvdepth) atomicAdd(out.dinvdepth + id, f[9]);
      } else {
        // The reference's helper: whole warp on one Gaussian -> reduce, else
        // per-lane atomics.
        const bool full = __match_any_sync(__activemask(), id) == 0xffffffffu;
        for (int q = 0; q < nf; ++q) {
          float v = f[q];
          if (full) {
#pragma unroll
            for (int off = 16; off; off >>= 1) v += __shfl_down_sync(0xffffffffu, v, off);
            if (lane == 0) atomicAdd(field_address(out, id, q), v);
          } else {
            atomicAdd(field_address(out, id, q), v);
          }
        }
      }
    }
  }
}

// Mode 2 with kPixelsPerThread pixels per thread: rows y, y + 16/k, ... of the
// tile. A thread keeps every pixel's back-to-front state; per Gaussian it adds
// its pixels' adjoints before the warp reduction, so each reduction covers
// 32 k pixels.
#ifndef CLAD3DGS_PIXELS_PER_THREAD
#define CLAD3DGS_PIXELS_PER_THREAD 4
#endif
constexpr int kPixelsPerThread = CLAD3DGS_PIXELS_PER_THREAD;
constexpr int kPairThreads = kTilePixels / kPixelsPerThread;

struct PixelState {
  bool inside;
  float fx, fy, T, T_final, dpix[3], dinv, bg_dot;
  uint32_t last, contributor;
  float acc[3], acc_inv, last_alpha, last_rgb[3], last_inv;
};

__device__ __forceinline__ void pixel_setup(PixelState& s, int px, int py, int width,
                                            int height, const float* __restrict__ final_t,
                                            const uint32_t* __restrict__ n_contrib,
                                            const float* __restrict__ dpixels,
                                            const float* __restrict__ dinvdepth_pixels,
                                            const float* __restrict__ bg) {
  s.inside = px < width && py < height;
  const int pix = py * width + px, hw = width * height;
  s.fx = (float)px;
  s.fy = (float)py;
  s.T_final = s.inside ? final_t[pix] : 0.f;
  s.T = s.T_final;
  s.last = s.inside ? n_contrib[pix] : 0;
  s.dpix[0] = s.dpix[1] = s.dpix[2] = 0.f;
  s.dinv = 0.f;
  if (s.inside) {
    s.dpix[0] = dpixels[pix];
    s.dpix[1] = dpixels[hw + pix];
    s.dpix[2] = dpixels[2 * hw + pix];
    if (dinvdepth_pixels) s.dinv = dinvdepth_pixels[pix];
  }
  s.bg_dot = bg[0] * s.dpix[0] + bg[1] * s.dpix[1] + bg[2] * s.dpix[2];
  s.acc[0] = s.acc[1] = s.acc[2] = 0.f;
  s.acc_inv = 0.f;
  s.last_alpha = 0.f;
  s.last_rgb[0] = s.last_rgb[1] = s.last_rgb[2] = 0.f;
  s.last_inv = 0.f;
}

// One (pixel, Gaussian) step of the walk: the same arithmetic as the one-pixel
// kernel, adding the pixel's ten adjoints into f; returns whether it contributed.
__device__ __forceinline__ bool pixel_step(PixelState& s, float2 xy, float4 co,
                                           const float* rgb3, float inv, float ddx,
                                           float ddy, float f[16]) {
  --s.contributor;
  bool contrib = s.inside && s.contributor < s.last;
  const float dx = xy.x - s.fx, dy = xy.y - s.fy;
  const float power = -0.5f * (co.x * dx * dx + co.z * dy * dy) - co.y * dx * dy;
  contrib = contrib && power <= 0.f;
  const float G = __expf(power);
  const float alpha = fminf(kMaxAlpha, co.w * G);
  contrib = contrib && alpha >= kMinAlpha;
  if (contrib) {
    const float inv_keep = 1.f / (1.f - alpha);
    s.T = s.T * inv_keep;
    const float w = alpha * s.T;
    float dl_dalpha = 0.f;
#pragma unroll
    for (int ch = 0; ch < 3; ++ch) {
      const float cc = rgb3[ch];
      s.acc[ch] = s.last_alpha * s.last_rgb[ch] + (1.f - s.last_alpha) * s.acc[ch];
      s.last_rgb[ch] = cc;
      dl_dalpha += (cc - s.acc[ch]) * s.dpix[ch];
      f[ch] += w * s.dpix[ch];
    }
    s.acc_inv = s.last_alpha * s.last_inv + (1.f - s.last_alpha) * s.acc_inv;
    s.last_inv = inv;
    dl_dalpha += (inv - s.acc_inv) * s.dinv;
    f[9] += w * s.dinv;
    dl_dalpha *= s.T;
    s.last_alpha = alpha;
    dl_dalpha += (-s.T_final * inv_keep) * s.bg_dot;
    const float dl_dg = co.w * dl_dalpha;
    const float gdx = G * dx, gdy = G * dy;
    const float dg_ddx = -gdx * co.x - gdy * co.y;
    const float dg_ddy = -gdy * co.z - gdx * co.y;
    f[3] += dl_dg * dg_ddx * ddx;
    f[4] += dl_dg * dg_ddy * ddy;
    f[5] += -0.5f * gdx * dx * dl_dg;
    f[6] += -0.5f * gdx * dy * dl_dg;
    f[7] += -0.5f * gdy * dy * dl_dg;
    f[8] += G * dl_dalpha;
  }
  return contrib;
}

__global__ void __launch_bounds__(kPairThreads)
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
  __shared__ uint32_t s_id[kBatch];
  __shared__ uint32_t s_last_max;
  __shared__ float2 s_xy[kBatch];
  __shared__ float4 s_co[kBatch];
  __shared__ float s_rgb[3 * kBatch];
  __shared__ float s_inv[kBatch];
  PixelState st[kPixelsPerThread];
  uint32_t my_last = 0;
#pragma unroll
  for (int r = 0; r < kPixelsPerThread; ++r) {
    pixel_setup(st[r], px, py + r * (kTileY / kPixelsPerThread), width, height, final_t,
                n_contrib, dpixels, dinvdepth_pixels, bg);
    my_last = max(my_last, st[r].last);
  }
  // Start at the tile's largest last-contributor index (see the one-pixel kernel).
  if (threadIdx.x == 0) s_last_max = 0;
  __syncthreads();
  const uint32_t warp_max = __reduce_max_sync(0xffffffffu, my_last);
  if (lane == 0) atomicMax(&s_last_max, warp_max);
  __syncthreads();
  const int todo = int(s_last_max);
#pragma unroll
  for (int r = 0; r < kPixelsPerThread; ++r) st[r].contributor = todo;
  const float ddx = 0.5f * width, ddy = 0.5f * height;
  const int nf = out.dinvdepth ? 10 : 9;
  for (int base = 0; base < todo; base += kBatch) {
    __syncthreads();
#pragma unroll
    for (int h = 0; h < kPixelsPerThread; ++h) {
      const int slot = threadIdx.x + h * kPairThreads;
      const int k = base + slot;
      if (k < todo) {
        const uint32_t id = point_list[range.x + todo - k - 1];
        s_id[slot] = id;
        s_xy[slot] = mean2d[id];
        s_co[slot] = conic_opacity[id];
        s_rgb[3 * slot] = rgb[3 * id];
        s_rgb[3 * slot + 1] = rgb[3 * id + 1];
        s_rgb[3 * slot + 2] = rgb[3 * id + 2];
        s_inv[slot] = 1.f / depth[id];
      }
    }
    __syncthreads();
    const int count = min(kBatch, todo - base);
    for (int j = 0; j < count; ++j) {
      float f[16];
#pragma unroll
      for (int q = 0; q < 16; ++q) f[q] = 0.f;
      const float2 xy = s_xy[j];
      const float4 co = s_co[j];
      const float* rgb3 = s_rgb + 3 * j;
      const float inv = s_inv[j];
      bool any = false;
#pragma unroll
      for (int r = 0; r < kPixelsPerThread; ++r)
        any = pixel_step(st[r], xy, co, rgb3, inv, ddx, ddy, f) || any;
      if (!__any_sync(0xffffffffu, any)) continue;
      const float total = transpose_reduce(f, lane);
      const int q = (lane >> 1) & 15;
      if ((lane & 1) == 0 && q < nf) atomicAdd(field_address(out, s_id[j], q), total);
    }
  }
}

// ---------------------------------------------------------------------------
// Geometry backward: one thread per Gaussian.

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
  float a0, b, c0;
  covariance2d(J, cov, a0, b, c0);
  const float a = a0 + kLowPass, c = c0 + kLowPass;
  const float det0 = a0 * c0 - b * b;
  const float det = a * c - b * b;
  // Opacity: the renderer used opacity * s with s = sqrt(max(2.5e-5, det0/det)).
  float dl_da = 0.f, dl_db = 0.f, dl_dc = 0.f;
  const float dop_scaled = o.dopacity[i];
  if (antialiasing) {
    const float r = det0 / det;
    const float s = sqrtf(fmaxf(0.000025f, r));
    o.dopacity[i] = dop_scaled * s;
    if (r > 0.000025f) {
      const float dl_ds = dop_scaled * opacities[i];
      const float dl_dr = dl_ds * 0.5f / s;
      const float id2 = 1.f / (det * det);
      // r = det0 / det; d det0 = (c0, -2b, a0), d det = (c, -2b, a) wrt (a0, b, c0)
      dl_da += dl_dr * (c0 * det - det0 * c) * id2;
      dl_db += dl_dr * (-2.f * b * det + 2.f * b * det0) * id2;
      dl_dc += dl_dr * (a0 * det - det0 * a) * id2;
    }
  }
  // Conic = inverse of [[a, b], [b, c]]; dconic.y holds half the adjoint of the
  // off-diagonal value (each symmetric entry receives it).
  const float* dq = o.dconic + 4 * i;
  const float gx = dq[0], gy2 = dq[1], gz = dq[3];
  const float id2 = 1.f / (det * det + 0.0000001f);
  if (id2 != 0.f) {
    dl_da += id2 * (-c * c * gx + 2.f * b * c * gy2 + (det - a * c) * gz);
    dl_dc += id2 * (-a * a * gz + 2.f * a * b * gy2 + (det - a * c) * gx);
    dl_db += id2 * 2.f * (b * c * gx - (det + 2.f * b * b) * gy2 + a * b * gz);
  }
  // Screen covariance A Sigma A^T -> Sigma (six unique entries).
  const float* A0 = J.A;
  const float* A1 = J.A + 3;
  float dcov[6];
  {
    int k = 0;
    for (int r = 0; r < 3; ++r)
      for (int s = r; s < 3; ++s, ++k) {
        const float mul = r == s ? 1.f : 2.f;
        const float sym_b = r == s ? A0[r] * A1[r] : A0[r] * A1[s] + A0[s] * A1[r];
        dcov[k] = mul * (A0[r] * A0[s] * dl_da + A1[r] * A1[s] * dl_dc) + sym_b * dl_db;
      }
  }
#pragma unroll
  for (int k = 0; k < 6; ++k) o.dcov3d[6 * i + k] = dcov[k];
  // Through the projection Jacobian to the camera-space mean.
  const float S[9] = {cov[0], cov[1], cov[2], cov[1], cov[3], cov[4], cov[2], cov[4], cov[5]};
  float sa0[3], sa1[3];
#pragma unroll
  for (int k = 0; k < 3; ++k) {
    sa0[k] = S[3 * k] * A0[0] + S[3 * k + 1] * A0[1] + S[3 * k + 2] * A0[2];
    sa1[k] = S[3 * k] * A1[0] + S[3 * k + 1] * A1[1] + S[3 * k + 2] * A1[2];
  }
  float dA0[3], dA1[3];
#pragma unroll
  for (int k = 0; k < 3; ++k) {
    dA0[k] = 2.f * dl_da * sa0[k] + dl_db * sa1[k];
    dA1[k] = dl_db * sa0[k] + 2.f * dl_dc * sa1[k];
  }
  // A = J W: dJ = dA W^T; J00 = fx/z, J02 = -fx tx/z^2, J11 = fy/z, J12 = -fy ty/z^2.
  float dJ00 = 0.f, dJ02 = 0.f, dJ11 = 0.f, dJ12 = 0.f;
#pragma unroll
  for (int col = 0; col < 3; ++col) {
    dJ00 += dA0[col] * cam.view[4 * col + 0];
    dJ02 += dA0[col] * cam.view[4 * col + 2];
    dJ11 += dA1[col] * cam.view[4 * col + 1];
    dJ12 += dA1[col] * cam.view[4 * col + 2];
  }
  const float iz = 1.f / J.tz, iz2 = iz * iz, iz3 = iz2 * iz;
  const float dtx = (J.clamp_x ? 0.f : 1.f) * -cam.fx * iz2 * dJ02;
  const float dty = (J.clamp_y ? 0.f : 1.f) * -cam.fy * iz2 * dJ12;
  float dtz = -cam.fx * iz2 * dJ00 - cam.fy * iz2 * dJ11 + 2.f * cam.fx * J.tx * iz3 * dJ02 +
              2.f * cam.fy * J.ty * iz3 * dJ12;
  if (o.dinvdepth) dtz += -o.dinvdepth[i] * iz2;
  // Camera-space -> world: t = W p + b, so dp = W^T dt.
  float dm[3];
#pragma unroll
  for (int k = 0; k < 3; ++k)
    dm[k] = cam.view[4 * k + 0] * dtx + cam.view[4 * k + 1] * dty + cam.view[4 * k + 2] * dtz;
  // Screen mean (NDC adjoint) -> world mean through the projective divide.
  {
    const float hw = affine_w(cam.proj, p);
    const Vec3 h = affine3(cam.proj, p);
    const float iw = 1.f / (hw + 0.0000001f);
    const float gxn = o.dmean2d[3 * i], gyn = o.dmean2d[3 * i + 1];
    const float mx = h.x * iw * iw, my = h.y * iw * iw;
#pragma unroll
    for (int k = 0; k < 3; ++k) {
      const float pk3 = cam.proj[4 * k + 3];
      dm[k] += (cam.proj[4 * k + 0] * iw - pk3 * mx) * gxn +
               (cam.proj[4 * k + 1] * iw - pk3 * my) * gyn;
    }
  }
  // (The SH colour's share of dmeans, the view direction's adjoint, is added
  // by sh_backward_kernel afterwards.)
#pragma unroll
  for (int k = 0; k < 3; ++k) o.dmeans[3 * i + k] += dm[k];
  // Sigma = M M^T, M = R diag(s): dM = 2 G M with G the symmetric adjoint.
  if (!cov3d_precomp) {
    const float G[9] = {dcov[0], 0.5f * dcov[1], 0.5f * dcov[2], 0.5f * dcov[1], dcov[3],
                        0.5f * dcov[4], 0.5f * dcov[2], 0.5f * dcov[4], dcov[5]};
    const float s[3] = {scale_modifier * scales[3 * i], scale_modifier * scales[3 * i + 1],
                        scale_modifier * scales[3 * i + 2]};
    const float q[4] = {rotations[4 * i], rotations[4 * i + 1], rotations[4 * i + 2],
                        rotations[4 * i + 3]};
    float R[9];
    rotation(q, R);
    float M[9], dM[9];
#pragma unroll
    for (int r = 0; r < 3; ++r)
#pragma unroll
      for (int col = 0; col < 3; ++col) M[3 * r + col] = R[3 * r + col] * s[col];
#pragma unroll
    for (int r = 0; r < 3; ++r)
#pragma unroll
      for (int col = 0; col < 3; ++col)
        dM[3 * r + col] =
            2.f * (G[3 * r] * M[col] + G[3 * r + 1] * M[3 + col] + G[3 * r + 2] * M[6 + col]);
    // M_rc = R_rc s_c
#pragma unroll
    for (int col = 0; col < 3; ++col)
      o.dscales[3 * i + col] =
          scale_modifier * (dM[col] * R[col] + dM[3 + col] * R[3 + col] + dM[6 + col] * R[6 + col]);
    float dR[9];
#pragma unroll
    for (int r = 0; r < 3; ++r)
#pragma unroll
      for (int col = 0; col < 3; ++col) dR[3 * r + col] = dM[3 * r + col] * s[col];
    const float w = q[0], x = q[1], y = q[2], z = q[3];
    // dR/dq for R(w, x, y, z) of the rotation() above.
    o.drotations[4 * i + 0] = 2.f * (-z * dR[1] + y * dR[2] + z * dR[3] - x * dR[5] -
                                     y * dR[6] + x * dR[7]);
    o.drotations[4 * i + 1] = 2.f * (y * dR[1] + z * dR[2] + y * dR[3] - 2.f * x * dR[4] -
                                     w * dR[5] + z * dR[6] + w * dR[7] - 2.f * x * dR[8]);
    o.drotations[4 * i + 2] = 2.f * (-2.f * y * dR[0] + x * dR[1] + w * dR[2] + x * dR[3] +
                                     z * dR[5] - w * dR[6] + z * dR[7] - 2.f * y * dR[8]);
    o.drotations[4 * i + 3] = 2.f * (-2.f * z * dR[0] - w * dR[1] + x * dR[2] + w * dR[3] -
                                     2.f * z * dR[4] + y * dR[5] + x * dR[6] + y * dR[7]);
  }
}

// SH colour of every drawn Gaussian (radius > 0): colour + 0.5, clamped at 0,
// with the clamp flags the backward reads.
__global__ void __launch_bounds__(32 * kShWarps)
    sh_colour_kernel(int P, int degree, const float* __restrict__ means, ShSource sh,
                     const float* __restrict__ campos, GeomState g) {
  __shared__ float rows[kShWarps][32 * kShRow];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  float* blk = rows[warp];
  const int i0 = (blockIdx.x * kShWarps + warp) * 32;
  if (i0 >= P) return;  // whole warp
  const int n = min(32, P - i0);
  stage_coefficients(sh, i0, n, lane, blk);
  __syncwarp();
  const int i = i0 + lane;
  if (lane >= n || g.radii[i] <= 0) return;
  const Direction d = make_direction(means[3 * i], means[3 * i + 1], means[3 * i + 2],
                                     campos[0], campos[1], campos[2]);
  float rgb[3] = {0.f, 0.f, 0.f};
  colour_terms<0>(d, RowSource{blk + lane * kShRow}, i, (degree + 1) * (degree + 1), rgb);
#pragma unroll
  for (int k = 0; k < 3; ++k) {
    const float v = rgb[k] + 0.5f;
    g.clamped[3 * i + k] = v < 0.f;
    g.rgb[3 * i + k] = fmaxf(v, 0.f);
  }
}

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
      const int warps = (P + 31) / 32;
      sh_colour_kernel<<<(warps + kShWarps - 1) / kShWarps, 32 * kShWarps, 0, stream>>>(
          P, degree, means, sh, campos, g);
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
