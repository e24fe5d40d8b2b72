// Kernels of the data-parallel training step (one camera view per GPU,
// parameters replicated on every GPU, Adam moments sharded by Gaussian index):
//
//   activate_kernel      raw log-scale / quaternion / opacity logit -> exp,
//                        normalised quaternion, sigmoid, and the saved norm
//                        the quaternion VJP needs (activation.py:24-37).
//   l1_loss_kernel       mean absolute error of the rendered image and its
//                        gradient sign(d) / n.
//   shard_update_kernel  the exchange and the optimizer in one pass: for the
//                        Gaussians this GPU owns it reads the per-view
//                        gradients of every GPU (peer loads over NVLink, in
//                        rank order, so the sum is deterministic), applies the
//                        activation VJPs, runs torch-fused Adam with the
//                        owner's moments, and stores the updated parameters
//                        into every GPU's replica (peer stores). It replaces
//                        reduce-scatter -> Adam -> all-gather. With one source
//                        and one replica it is the local update of a shard
//                        whose gradients were reduced by a collective.
//
// Gradient groups (per Gaussian): xyz 3, SH 48 ([16][3], coefficient 0 is
// f_dc, 1..15 f_rest), scaling 3, rotation 4, opacity 1 = 59 floats. Every
// group is its own [N][k] array, so the owned range of a group is one
// contiguous span and moves as float4 chunks.
#include <cuda_runtime.h>

#include <cstdint>
#include <cstring>
#include <string>

#include "clad3dgs_b200.h"
#include "gaussian_math.cuh"

namespace clad3dgs {
int fail(int code, const std::string& message);  // gaussian_step.cu
}

namespace clad3dgs {
namespace train {

constexpr int kGroups = CLAD3DGS_SHARD_GROUPS;
constexpr int kMaxRanks = CLAD3DGS_MAX_RANKS;
constexpr int kThreads = 256;

__host__ __device__ constexpr int group_width(int g) {
  return g == 0 ? 3 : g == 1 ? 48 : g == 2 ? 3 : g == 3 ? 4 : 1;
}

__device__ __forceinline__ float4 add4(float4 a, float4 b) {
  return make_float4(a.x + b.x, a.y + b.y, a.z + b.z, a.w + b.w);
}

__global__ void __launch_bounds__(kThreads)
    activate_kernel(int64_t n, const float* __restrict__ scaling_raw,
                    const float4* __restrict__ rotation_raw,
                    const float* __restrict__ opacity_raw, float* __restrict__ scaling,
                    float4* __restrict__ rotation, float* __restrict__ opacity,
                    float* __restrict__ norms) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const float4 q = rotation_raw[i];
    const float norm = sqrtf(((q.x * q.x + q.y * q.y) + q.z * q.z) + q.w * q.w);
    const float d = fmaxf(norm, 1e-12f);
    rotation[i] = make_float4(q.x / d, q.y / d, q.z / d, q.w / d);
    norms[i] = norm;
#pragma unroll
    for (int k = 0; k < 3; ++k) scaling[3 * i + k] = expf(scaling_raw[3 * i + k]);
    opacity[i] = 1.f / (1.f + expf(-opacity_raw[i]));
  }
}

__global__ void __launch_bounds__(kThreads)
    l1_loss_kernel(int64_t n, const float* __restrict__ image,
                   const float* __restrict__ target, float scale,
                   float* __restrict__ dimage, float* __restrict__ loss) {
  float acc = 0.f;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const float d = image[i] - target[i];
    dimage[i] = d > 0.f ? scale : (d < 0.f ? -scale : 0.f);
    acc += fabsf(d);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
  __shared__ float partial[kThreads / 32];
  if ((threadIdx.x & 31) == 0) partial[threadIdx.x >> 5] = acc;
  __syncthreads();
  if (threadIdx.x == 0) {
    float s = 0.f;
#pragma unroll
    for (int w = 0; w < kThreads / 32; ++w) s += partial[w];
    atomicAdd(loss, s * scale);
  }
}

int blocks_for(int64_t work);

struct ShardParams {
  int64_t begin, end, grad_origin;
  int64_t chunk_begin;  // first float4 chunk updated here (past xyz and SH in seed form)
  int ranks, local;
  const float* grads[kMaxRanks][kGroups];
  float* params[kMaxRanks][kGroups];
  float* first[kGroups];
  float* second[kGroups];
  const float* saved_scaling;
  const float* saved_opacity;
  const float* saved_norm;
  float step[kGroups + 1];  // xyz, f_dc, f_rest, scaling, rotation, opacity
  double inv_bias2;
};

template <int R>
__global__ void __launch_bounds__(kThreads, R <= 2 ? 4 : 3)
    shard_update_kernel(const __grid_constant__ ShardParams a) {
  const int64_t n = a.end - a.begin;  // a multiple of 4
  // Chunk boundaries of the five groups (float4 chunks of the owned spans).
  const int64_t c0 = n * 3 / 4, c1 = c0 + n * 12, c2 = c1 + n * 3 / 4, c3 = c2 + n,
                c4 = c3 + n / 4;
  for (int64_t c = a.chunk_begin + blockIdx.x * (int64_t)blockDim.x + threadIdx.x; c < c4;
       c += (int64_t)gridDim.x * blockDim.x) {
    int g;
    int64_t local;
    if (c < c0) {
      g = 0, local = c;
    } else if (c < c1) {
      g = 1, local = c - c0;
    } else if (c < c2) {
      g = 2, local = c - c1;
    } else if (c < c3) {
      g = 3, local = c - c2;
    } else {
      g = 4, local = c - c3;
    }
    const int k = group_width(g);
    const int64_t elem = a.begin * k + 4 * local;       // index into full arrays
    const int64_t gelem = elem - a.grad_origin * k;     // index into gradients
    const int64_t melem = 4 * local;                    // index into moments
    // All sources first (independent loads, many in flight over NVLink), then
    // the sum in rank order.
    float4 t[R];
#pragma unroll
    for (int q = 0; q < R; ++q)
      t[q] = __ldcs(reinterpret_cast<const float4*>(a.grads[q][g] + gelem));
    float4 grad = t[0];
#pragma unroll
    for (int q = 1; q < R; ++q) grad = add4(grad, t[q]);
    float4 p = *reinterpret_cast<const float4*>(a.params[a.local][g] + elem);
    float4 m = *reinterpret_cast<const float4*>(a.first[g] + melem);
    float4 v = *reinterpret_cast<const float4*>(a.second[g] + melem);
    // Activation VJPs (controls/ManualActivations.cu:20-36, 94-100) with the
    // values saved by the forward activation.
    if (g == 2) {
      const float4 s = *reinterpret_cast<const float4*>(a.saved_scaling + elem);
      grad = make_float4(s.x * grad.x, s.y * grad.y, s.z * grad.z, s.w * grad.w);
    } else if (g == 4) {
      const float4 s = *reinterpret_cast<const float4*>(a.saved_opacity + elem);
      grad = make_float4((s.x * (1.f - s.x)) * grad.x, (s.y * (1.f - s.y)) * grad.y,
                         (s.z * (1.f - s.z)) * grad.z, (s.w * (1.f - s.w)) * grad.w);
    } else if (g == 3) {
      const float q[4] = {p.x, p.y, p.z, p.w};
      const float s[4] = {grad.x, grad.y, grad.z, grad.w};
      float out[4];
      quaternion_vjp(q, s, a.saved_norm[elem / 4], out);
      grad = make_float4(out[0], out[1], out[2], out[3]);
    }
    const float gv[4] = {grad.x, grad.y, grad.z, grad.w};
    float pv[4] = {p.x, p.y, p.z, p.w}, mv[4] = {m.x, m.y, m.z, m.w},
          vv[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      float step;
      if (g == 1)
        step = (elem + j) % 48 < 3 ? a.step[1] : a.step[2];
      else
        step = a.step[g == 0 ? 0 : g + 1];
      torch_adam(pv[j], mv[j], vv[j], gv[j], step, a.inv_bias2);
    }
    *reinterpret_cast<float4*>(a.first[g] + melem) = make_float4(mv[0], mv[1], mv[2], mv[3]);
    *reinterpret_cast<float4*>(a.second[g] + melem) = make_float4(vv[0], vv[1], vv[2], vv[3]);
    const float4 out = make_float4(pv[0], pv[1], pv[2], pv[3]);
#pragma unroll
    for (int q = 0; q < R; ++q) __stcs(reinterpret_cast<float4*>(a.params[q][g] + elem), out);
  }
  // Make the peer stores visible system-wide before the kernel retires.
  if (R > 1) __threadfence_system();
}

// One float4 chunk of the owned spans: where it lives and everything loaded
// for it (every source's gradients, the parameters, both moments, the saved
// activation value).
template <int R>
struct Chunk {
  int g;
  int64_t elem, melem;  // index into full arrays / into the moments
  float4 t[R], p, m, v, s;
};

template <int R>
__device__ __forceinline__ void load_chunk(const ShardParams& a, int64_t c, int64_t n,
                                           Chunk<R>& x) {
  // Chunk boundaries of the five groups (float4 chunks of the owned spans).
  const int64_t c0 = n * 3 / 4, c1 = c0 + n * 12, c2 = c1 + n * 3 / 4, c3 = c2 + n;
  int64_t local;
  if (c < c0) {
    x.g = 0, local = c;
  } else if (c < c1) {
    x.g = 1, local = c - c0;
  } else if (c < c2) {
    x.g = 2, local = c - c1;
  } else if (c < c3) {
    x.g = 3, local = c - c2;
  } else {
    x.g = 4, local = c - c3;
  }
  const int k = group_width(x.g);
  x.elem = a.begin * k + 4 * local;
  x.melem = 4 * local;
  const int64_t gelem = x.elem - a.grad_origin * k;
#pragma unroll
  for (int q = 0; q < R; ++q)
    x.t[q] = __ldcs(reinterpret_cast<const float4*>(a.grads[q][x.g] + gelem));
  x.p = *reinterpret_cast<const float4*>(a.params[a.local][x.g] + x.elem);
  x.m = *reinterpret_cast<const float4*>(a.first[x.g] + x.melem);
  x.v = *reinterpret_cast<const float4*>(a.second[x.g] + x.melem);
  if (x.g == 2) x.s = *reinterpret_cast<const float4*>(a.saved_scaling + x.elem);
  else if (x.g == 4) x.s = *reinterpret_cast<const float4*>(a.saved_opacity + x.elem);
  else if (x.g == 3) x.s.x = a.saved_norm[x.elem / 4];
}

template <int R>
__device__ __forceinline__ void update_chunk(const ShardParams& a, const Chunk<R>& x) {
  // The sum in rank order.
  float4 grad = x.t[0];
#pragma unroll
  for (int q = 1; q < R; ++q) grad = add4(grad, x.t[q]);
  // Activation VJPs (controls/ManualActivations.cu:20-36, 94-100) with the
  // values saved by the forward activation.
  if (x.g == 2) {
    grad = make_float4(x.s.x * grad.x, x.s.y * grad.y, x.s.z * grad.z, x.s.w * grad.w);
  } else if (x.g == 4) {
    const float4 s = x.s;
    grad = make_float4((s.x * (1.f - s.x)) * grad.x, (s.y * (1.f - s.y)) * grad.y,
                       (s.z * (1.f - s.z)) * grad.z, (s.w * (1.f - s.w)) * grad.w);
  } else if (x.g == 3) {
    const float q[4] = {x.p.x, x.p.y, x.p.z, x.p.w};
    const float sd[4] = {grad.x, grad.y, grad.z, grad.w};
    float out[4];
    quaternion_vjp(q, sd, x.s.x, out);
    grad = make_float4(out[0], out[1], out[2], out[3]);
  }
  const float gv[4] = {grad.x, grad.y, grad.z, grad.w};
  float pv[4] = {x.p.x, x.p.y, x.p.z, x.p.w}, mv[4] = {x.m.x, x.m.y, x.m.z, x.m.w},
        vv[4] = {x.v.x, x.v.y, x.v.z, x.v.w};
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    float step;
    if (x.g == 1)
      step = (x.elem + j) % 48 < 3 ? a.step[1] : a.step[2];
    else
      step = a.step[x.g == 0 ? 0 : x.g + 1];
    torch_adam(pv[j], mv[j], vv[j], gv[j], step, a.inv_bias2);
  }
  *reinterpret_cast<float4*>(a.first[x.g] + x.melem) = make_float4(mv[0], mv[1], mv[2], mv[3]);
  *reinterpret_cast<float4*>(a.second[x.g] + x.melem) = make_float4(vv[0], vv[1], vv[2], vv[3]);
  const float4 out = make_float4(pv[0], pv[1], pv[2], pv[3]);
#pragma unroll
  for (int q = 0; q < R; ++q) __stcs(reinterpret_cast<float4*>(a.params[q][x.g] + x.elem), out);
}

// With peers: grid-stride over the chunks, each thread loading its next chunk
// before it updates the current one, so the loads over NVLink stay in flight
// during the Adam arithmetic (measured faster with 2 GPUs; on one GPU the
// plain kernel above, with more resident threads, is faster).
template <int R>
__global__ void __launch_bounds__(kThreads, R <= 4 ? 3 : 2)
    shard_update_prefetch_kernel(const __grid_constant__ ShardParams a) {
  const int64_t n = a.end - a.begin;  // a multiple of 4
  const int64_t chunks = n * 59 / 4;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  int64_t c = a.chunk_begin + blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (c >= chunks) return;
  Chunk<R> cur;
  load_chunk<R>(a, c, n, cur);
  for (;;) {
    const int64_t next = c + stride;
    if (next < chunks) {
      Chunk<R> nx;
      load_chunk<R>(a, next, n, nx);
      update_chunk<R>(a, cur);
      cur = nx;
      c = next;
    } else {
      update_chunk<R>(a, cur);
      break;
    }
  }
  // Make the peer stores visible system-wide before the kernel retires.
  if (R > 1) __threadfence_system();
}

template <int R>
cudaError_t launch_shard_update(const ShardParams& p, int64_t chunks, cudaStream_t stream) {
  const int blocks = blocks_for(chunks - p.chunk_begin);
  if constexpr (R == 1)
    shard_update_kernel<R><<<blocks, kThreads, 0, stream>>>(p);
  else
    shard_update_prefetch_kernel<R><<<blocks, kThreads, 0, stream>>>(p);
  return cudaGetLastError();
}

int blocks_for(int64_t work) {
  int device = 0, sms = 148;
  cudaGetDevice(&device);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
  const int64_t need = (work + kThreads - 1) / kThreads;
  const int64_t cap = int64_t(sms) * (2048 / kThreads);
  return int(need < cap ? (need > 0 ? need : 1) : cap);
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

int shard_seed_update(const clad3dgs_shard_update_args& x, cudaStream_t stream);  // shard_sh.cu

}  // namespace train
}  // namespace clad3dgs

using namespace clad3dgs;
using namespace clad3dgs::train;

extern "C" int clad3dgs_activate(int64_t n, const float* scaling_raw,
                                 const float* rotation_raw, const float* opacity_raw,
                                 float* scaling, float* rotation, float* opacity,
                                 float* norms, cudaStream_t stream) {
  if (n < 0) return fail(CLAD3DGS_INVALID_ARGUMENT, "activate: negative count");
  if (n == 0) return CLAD3DGS_OK;
  if (!scaling_raw || !rotation_raw || !opacity_raw || !scaling || !rotation || !opacity ||
      !norms)
    return fail(CLAD3DGS_INVALID_ARGUMENT, "activate: null pointer");
  if (!aligned16(rotation_raw) || !aligned16(rotation))
    return fail(CLAD3DGS_INVALID_ARGUMENT, "activate: quaternions must be 16-byte aligned");
  activate_kernel<<<blocks_for(n), kThreads, 0, stream>>>(
      n, scaling_raw, reinterpret_cast<const float4*>(rotation_raw), opacity_raw, scaling,
      reinterpret_cast<float4*>(rotation), opacity, norms);
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? CLAD3DGS_OK
                          : fail(CLAD3DGS_CUDA_ERROR, std::string("activate: ") +
                                                          cudaGetErrorString(e));
}

extern "C" int clad3dgs_l1_loss(int64_t n, const float* image, const float* target,
                                float* dimage, float* loss, cudaStream_t stream) {
  if (n <= 0) return fail(CLAD3DGS_INVALID_ARGUMENT, "l1 loss: empty image");
  if (!image || !target || !dimage || !loss)
    return fail(CLAD3DGS_INVALID_ARGUMENT, "l1 loss: null pointer");
  l1_loss_kernel<<<blocks_for(n), kThreads, 0, stream>>>(n, image, target, 1.f / float(n),
                                                         dimage, loss);
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? CLAD3DGS_OK
                          : fail(CLAD3DGS_CUDA_ERROR, std::string("l1 loss: ") +
                                                          cudaGetErrorString(e));
}

extern "C" int clad3dgs_shard_update(const clad3dgs_shard_update_args* args,
                                     cudaStream_t stream) {
  if (!args) return fail(CLAD3DGS_INVALID_ARGUMENT, "shard update: null arguments");
  const clad3dgs_shard_update_args& x = *args;
  if (x.ranks < 1 || x.ranks > kMaxRanks)
    return fail(CLAD3DGS_INVALID_ARGUMENT, "shard update: ranks must be 1..8");
  if (x.local < 0 || x.local >= x.ranks)
    return fail(CLAD3DGS_INVALID_ARGUMENT, "shard update: local replica out of range");
  if (x.begin < 0 || x.end < x.begin || x.begin % 4 || x.end % 4 || x.grad_origin % 4 ||
      x.grad_origin > x.begin)
    return fail(CLAD3DGS_INVALID_ARGUMENT,
                "shard update: range must be ordered multiples of 4 at or after grad_origin");
  if (!(x.bias1 > 0.f) || !(x.bias2_sqrt > 0.f))
    return fail(CLAD3DGS_INVALID_ARGUMENT, "shard update: bias corrections must be positive");
  if (x.end == x.begin) return CLAD3DGS_OK;
  const bool seeded = x.seeds[0] != nullptr;
  ShardParams p{};
  p.begin = x.begin;
  p.end = x.end;
  p.grad_origin = x.grad_origin;
  p.ranks = x.ranks;
  p.local = x.local;
  for (int g = 0; g < kGroups; ++g) {
    for (int q = 0; q < x.ranks; ++q) {
      const bool unused = seeded && g == 1;  // the SH gradients come from the seeds
      if ((!unused && (!x.grads[q][g] || !aligned16(x.grads[q][g]))) || !x.params[q][g] ||
          !aligned16(x.params[q][g]))
        return fail(CLAD3DGS_INVALID_ARGUMENT,
                    "shard update: gradient and parameter arrays must be non-null and "
                    "16-byte aligned");
      p.grads[q][g] = x.grads[q][g];
      p.params[q][g] = x.params[q][g];
    }
    if (!x.first[g] || !x.second[g] || !aligned16(x.first[g]) || !aligned16(x.second[g]))
      return fail(CLAD3DGS_INVALID_ARGUMENT,
                  "shard update: moments must be non-null and 16-byte aligned");
    p.first[g] = x.first[g];
    p.second[g] = x.second[g];
  }
  if (!x.saved_scaling || !x.saved_opacity || !x.saved_norm || !aligned16(x.saved_scaling) ||
      !aligned16(x.saved_opacity))
    return fail(CLAD3DGS_INVALID_ARGUMENT,
                "shard update: saved activations must be non-null and 16-byte aligned");
  p.saved_scaling = x.saved_scaling;
  p.saved_opacity = x.saved_opacity;
  p.saved_norm = x.saved_norm;
  for (int r = 0; r < kGroups + 1; ++r) p.step[r] = float(x.rates[r] / double(x.bias1));
  p.inv_bias2 = 1.0 / double(x.bias2_sqrt);
  const int64_t n = x.end - x.begin;
  const int64_t chunks = n * 59 / 4;
  if (seeded) {
    const int status = shard_seed_update(x, stream);
    if (status != CLAD3DGS_OK) return status;
    p.chunk_begin = n * 3 / 4 + n * 12;  // past the xyz and SH chunks
  }
  cudaError_t e = cudaSuccess;
  switch (x.ranks) {
    case 1: e = launch_shard_update<1>(p, chunks, stream); break;
    case 2: e = launch_shard_update<2>(p, chunks, stream); break;
    case 3: e = launch_shard_update<3>(p, chunks, stream); break;
    case 4: e = launch_shard_update<4>(p, chunks, stream); break;
    case 5: e = launch_shard_update<5>(p, chunks, stream); break;
    case 6: e = launch_shard_update<6>(p, chunks, stream); break;
    case 7: e = launch_shard_update<7>(p, chunks, stream); break;
    default: e = launch_shard_update<8>(p, chunks, stream); break;
  }
  return e == cudaSuccess ? CLAD3DGS_OK
                          : fail(CLAD3DGS_CUDA_ERROR, std::string("shard update: ") +
                                                          cudaGetErrorString(e));
}

// Device memory that other processes on this node can map (CUDA IPC): the
// replicated parameters and the per-view gradients of the peer exchange.
extern "C" int clad3dgs_ipc_alloc(size_t bytes, void** ptr, unsigned char* handle) {
  if (!ptr || !handle || bytes == 0)
    return fail(CLAD3DGS_INVALID_ARGUMENT, "ipc alloc: bad arguments");
  *ptr = nullptr;
  cudaError_t e = cudaMalloc(ptr, bytes);
  if (e != cudaSuccess)
    return fail(CLAD3DGS_CUDA_ERROR, std::string("ipc alloc: ") + cudaGetErrorString(e));
  e = cudaMemset(*ptr, 0, bytes);
  cudaIpcMemHandle_t h;
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, *ptr);
  if (e != cudaSuccess) {
    cudaFree(*ptr);
    *ptr = nullptr;
    return fail(CLAD3DGS_CUDA_ERROR, std::string("ipc alloc: ") + cudaGetErrorString(e));
  }
  static_assert(sizeof(h) == CLAD3DGS_IPC_HANDLE_BYTES, "IPC handle size");
  memcpy(handle, &h, sizeof(h));
  return CLAD3DGS_OK;
}

extern "C" int clad3dgs_ipc_free(void* ptr) {
  const cudaError_t e = cudaFree(ptr);
  return e == cudaSuccess ? CLAD3DGS_OK
                          : fail(CLAD3DGS_CUDA_ERROR, std::string("ipc free: ") +
                                                          cudaGetErrorString(e));
}

extern "C" int clad3dgs_ipc_open(const unsigned char* handle, void** ptr) {
  if (!ptr || !handle) return fail(CLAD3DGS_INVALID_ARGUMENT, "ipc open: bad arguments");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  const cudaError_t e = cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess);
  return e == cudaSuccess ? CLAD3DGS_OK
                          : fail(CLAD3DGS_CUDA_ERROR, std::string("ipc open: ") +
                                                          cudaGetErrorString(e));
}

extern "C" int clad3dgs_ipc_close(void* ptr) {
  const cudaError_t e = cudaIpcCloseMemHandle(ptr);
  return e == cudaSuccess ? CLAD3DGS_OK
                          : fail(CLAD3DGS_CUDA_ERROR, std::string("ipc close: ") +
                                                          cudaGetErrorString(e));
}
