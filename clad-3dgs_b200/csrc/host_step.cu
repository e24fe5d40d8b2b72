// Host-buffer entry of the fused per-Gaussian step.
//
// For callers whose Gaussians live in pinned host memory (the setting of the
// reference's CPU path): Gaussians are cut into chunks, and each chunk goes
// through copy-in -> fused kernel -> copy-out on three streams with NB staging
// sets, so the PCIe copy-in of chunk c+1, the kernel on chunk c and the
// copy-out of chunk c-1 overlap. One cudaMemcpyAsync per array and chunk.
#include <cstdint>
#include <cstring>
#include <mutex>
#include <string>

#include "clad3dgs_b200.h"

namespace {

constexpr int kSets = 3;              // staging sets in the workspace
constexpr size_t kAlign = 256;

size_t round_up(size_t v) { return (v + kAlign - 1) / kAlign * kAlign; }

// Per-Gaussian element counts of the staged arrays, in workspace order.
enum Slot : int {
  S_MEANS, S_RADII, S_CLAMPED, S_SEED, S_DM, S_DC, S_DC_M, S_DC_V, S_REST,
  S_REST_M, S_REST_V, S_ROT, S_ROT_M, S_ROT_V, S_SCL, S_SCL_M, S_SCL_V, S_OPA,
  S_OPA_M, S_OPA_V, S_SEED_ROT, S_SEED_SCL, S_SEED_OPA, S_NORM, S_EXPS, S_SIG,
  S_COUNT
};
constexpr int kSlotWidth[S_COUNT] = {3, 1, 3, 3, 3, 3, 3, 3, 45, 45, 45, 4, 4,
                                     4, 3, 3, 3, 1, 1, 1, 4, 3, 1, 1, 3, 1};
constexpr bool kSlotOut[S_COUNT] = {0, 0, 0, 0, 1, 1, 1, 1, 1, 1, 1, 1, 1,
                                    1, 1, 1, 1, 1, 1, 1, 0, 0, 0, 0, 0, 0};
size_t slot_elem(int s) { return s == S_CLAMPED ? 1 : 4; }

size_t set_bytes(int64_t chunk) {
  size_t total = 0;
  for (int s = 0; s < S_COUNT; ++s)
    total += round_up(size_t(chunk) * kSlotWidth[s] * slot_elem(s));
  return total;
}

struct Streams {
  cudaStream_t in = nullptr, run = nullptr, out = nullptr;
  cudaEvent_t start = nullptr, loaded[kSets] = {}, stepped[kSets] = {},
              drained[kSets] = {};
  bool ready = false;
};

std::mutex g_lock;
Streams g_streams[64];

cudaError_t streams_for_device(Streams** result) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  Streams& s = g_streams[dev & 63];
  if (!s.ready) {
    const unsigned f = cudaStreamNonBlocking;
    if ((e = cudaStreamCreateWithFlags(&s.in, f)) != cudaSuccess) return e;
    if ((e = cudaStreamCreateWithFlags(&s.run, f)) != cudaSuccess) return e;
    if ((e = cudaStreamCreateWithFlags(&s.out, f)) != cudaSuccess) return e;
    const unsigned ef = cudaEventDisableTiming;
    if ((e = cudaEventCreateWithFlags(&s.start, ef)) != cudaSuccess) return e;
    for (int k = 0; k < kSets; ++k) {
      if ((e = cudaEventCreateWithFlags(&s.loaded[k], ef)) != cudaSuccess) return e;
      if ((e = cudaEventCreateWithFlags(&s.stepped[k], ef)) != cudaSuccess) return e;
      if ((e = cudaEventCreateWithFlags(&s.drained[k], ef)) != cudaSuccess) return e;
    }
    s.ready = true;
  }
  *result = &s;
  return cudaSuccess;
}

}  // namespace

namespace clad3dgs {
int fail(int code, const std::string& message);  // gaussian_step.cu
}

extern "C" size_t clad3dgs_host_step_workspace(int64_t chunk_gaussians) {
  if (chunk_gaussians <= 0) return 0;
  return kSets * set_bytes(chunk_gaussians) + kAlign;  // + camera
}

extern "C" int clad3dgs_gaussian_step_host(
    int64_t n, int degree, const float* means_host, const int* radii_host,
    const bool* clamped_host, const float* camera_host, const float* seed_host,
    float* dm_host, float* dc_host, float* rest_host, float* dc_first_host,
    float* dc_second_host, float* rest_first_host, float* rest_second_host,
    TorchAdamConfig sh_config, float* const* parameters_host,
    const float* const* seeds_host, const float* const* saved_host,
    float* const* first_host, float* const* second_host, const double* rates,
    const float* bias1, const float* bias2, void* workspace_dev,
    size_t workspace_bytes, int64_t chunk_gaussians, cudaStream_t stream) {
  if (n <= 0) return CLAD3DGS_OK;
  if (degree < 0 || degree > 3 || chunk_gaussians <= 0 || chunk_gaussians % 64 ||
      workspace_bytes < clad3dgs_host_step_workspace(chunk_gaussians)) {
    return clad3dgs::fail(
        CLAD3DGS_INVALID_ARGUMENT,
        "host step needs degree 0..3, a chunk that is a positive multiple of 64 "
        "and clad3dgs_host_step_workspace(chunk) bytes of workspace");
  }
  std::lock_guard<std::mutex> guard(g_lock);
  Streams* ss = nullptr;
  cudaError_t e = streams_for_device(&ss);
  if (e != cudaSuccess) return clad3dgs::fail(CLAD3DGS_CUDA_ERROR, cudaGetErrorString(e));
  const void* host[S_COUNT] = {
      means_host,         radii_host,         clamped_host,
      seed_host,          dm_host,            dc_host,
      dc_first_host,      dc_second_host,     rest_host,
      rest_first_host,    rest_second_host,   parameters_host[0],
      first_host[0],      second_host[0],     parameters_host[1],
      first_host[1],      second_host[1],     parameters_host[2],
      first_host[2],      second_host[2],     seeds_host[0],
      seeds_host[1],      seeds_host[2],      saved_host[0],
      saved_host[1],      saved_host[2]};
  char* ws = static_cast<char*>(workspace_dev);
  float* camera_dev = reinterpret_cast<float*>(ws + kSets * set_bytes(chunk_gaussians));
  auto check = [&](cudaError_t err) {
    if (err != cudaSuccess && e == cudaSuccess) e = err;
  };
  check(cudaEventRecord(ss->start, stream));
  check(cudaStreamWaitEvent(ss->in, ss->start, 0));
  check(cudaStreamWaitEvent(ss->run, ss->start, 0));
  check(cudaStreamWaitEvent(ss->out, ss->start, 0));
  check(cudaMemcpyAsync(camera_dev, camera_host, 3 * sizeof(float),
                        cudaMemcpyHostToDevice, ss->in));
  const int64_t chunks = (n + chunk_gaussians - 1) / chunk_gaussians;
  for (int64_t c = 0; c < chunks && e == cudaSuccess; ++c) {
    const int set = int(c % kSets);
    const int64_t g0 = c * chunk_gaussians;
    const int64_t cnt = (n - g0) < chunk_gaussians ? (n - g0) : chunk_gaussians;
    char* dev[S_COUNT];
    char* cursor = ws + set * set_bytes(chunk_gaussians);
    for (int s = 0; s < S_COUNT; ++s) {
      dev[s] = cursor;
      cursor += round_up(size_t(chunk_gaussians) * kSlotWidth[s] * slot_elem(s));
    }
    // The staging set is free once the copy-out of chunk c - kSets finished.
    if (c >= kSets) check(cudaStreamWaitEvent(ss->in, ss->drained[set], 0));
    for (int s = 0; s < S_COUNT; ++s) {
      const size_t row = kSlotWidth[s] * slot_elem(s);
      check(cudaMemcpyAsync(dev[s], static_cast<const char*>(host[s]) + g0 * row,
                            size_t(cnt) * row, cudaMemcpyHostToDevice, ss->in));
    }
    check(cudaEventRecord(ss->loaded[set], ss->in));
    check(cudaStreamWaitEvent(ss->run, ss->loaded[set], 0));
    float* params[3] = {reinterpret_cast<float*>(dev[S_ROT]),
                        reinterpret_cast<float*>(dev[S_SCL]),
                        reinterpret_cast<float*>(dev[S_OPA])};
    float* firsts[3] = {reinterpret_cast<float*>(dev[S_ROT_M]),
                        reinterpret_cast<float*>(dev[S_SCL_M]),
                        reinterpret_cast<float*>(dev[S_OPA_M])};
    float* seconds[3] = {reinterpret_cast<float*>(dev[S_ROT_V]),
                         reinterpret_cast<float*>(dev[S_SCL_V]),
                         reinterpret_cast<float*>(dev[S_OPA_V])};
    const float* seeds[3] = {reinterpret_cast<float*>(dev[S_SEED_ROT]),
                             reinterpret_cast<float*>(dev[S_SEED_SCL]),
                             reinterpret_cast<float*>(dev[S_SEED_OPA])};
    const float* saved[3] = {reinterpret_cast<float*>(dev[S_NORM]),
                             reinterpret_cast<float*>(dev[S_EXPS]),
                             reinterpret_cast<float*>(dev[S_SIG])};
    const int status = clad3dgs_gaussian_step(
        cnt, degree, reinterpret_cast<float*>(dev[S_MEANS]),
        reinterpret_cast<int*>(dev[S_RADII]), nullptr,
        reinterpret_cast<bool*>(dev[S_CLAMPED]), camera_dev,
        reinterpret_cast<float*>(dev[S_SEED]), reinterpret_cast<float*>(dev[S_DM]),
        reinterpret_cast<float*>(dev[S_DC]), reinterpret_cast<float*>(dev[S_REST]),
        reinterpret_cast<float*>(dev[S_DC_M]), reinterpret_cast<float*>(dev[S_DC_V]),
        reinterpret_cast<float*>(dev[S_REST_M]),
        reinterpret_cast<float*>(dev[S_REST_V]), sh_config, params, seeds, saved,
        firsts, seconds, rates, bias1, bias2, ss->run);
    if (status != CLAD3DGS_OK) {
      cudaStreamSynchronize(ss->in);
      cudaStreamSynchronize(ss->run);
      cudaStreamSynchronize(ss->out);
      return status;
    }
    check(cudaEventRecord(ss->stepped[set], ss->run));
    check(cudaStreamWaitEvent(ss->out, ss->stepped[set], 0));
    for (int s = 0; s < S_COUNT; ++s) {
      if (!kSlotOut[s]) continue;
      const size_t row = kSlotWidth[s] * slot_elem(s);
      check(cudaMemcpyAsync(static_cast<char*>(const_cast<void*>(host[s])) + g0 * row,
                            dev[s], size_t(cnt) * row, cudaMemcpyDeviceToHost,
                            ss->out));
    }
    check(cudaEventRecord(ss->drained[set], ss->out));
  }
  cudaEvent_t done = ss->drained[(chunks - 1) % kSets];
  check(cudaStreamWaitEvent(stream, done, 0));
  check(cudaStreamSynchronize(stream));
  if (e != cudaSuccess) {
    cudaGetLastError();
    return clad3dgs::fail(CLAD3DGS_CUDA_ERROR, cudaGetErrorString(e));
  }
  return CLAD3DGS_OK;
}

// ---------------------------------------------------------------------------
// Allocation-free variant: the staging set lives in a fixed device array.

namespace {

// One staging set plus the camera, for callers that cannot allocate.
static __device__ __align__(256) unsigned char
    g_static_staging[CLAD3DGS_STATIC_STAGING_BYTES];

std::mutex g_static_lock;
void* g_static_address[64] = {};  // device address of g_static_staging, per device

// Largest multiple of 64 Gaussians whose staging set and camera fit the array.
// The results go back from the same slots the inputs came in, so a chunk needs
// the staged bytes once: start from the array size over the bytes per
// Gaussian and step down past the slot padding.
int64_t static_chunk_limit() {
  size_t per_gaussian = 0;
  for (int s = 0; s < S_COUNT; ++s) per_gaussian += kSlotWidth[s] * slot_elem(s);
  int64_t chunk = int64_t(CLAD3DGS_STATIC_STAGING_BYTES / per_gaussian) / 64 * 64;
  while (chunk > 0 && set_bytes(chunk) + kAlign > CLAD3DGS_STATIC_STAGING_BYTES)
    chunk -= 64;
  return chunk;
}

}  // namespace

extern "C" int clad3dgs_gaussian_step_host_static(
    int64_t n, int degree, const float* means_host, const int* radii_host,
    const bool* clamped_host, const float* camera_host, const float* seed_host,
    float* dm_host, float* dc_host, float* rest_host, float* dc_first_host,
    float* dc_second_host, float* rest_first_host, float* rest_second_host,
    TorchAdamConfig sh_config, float* const* parameters_host,
    const float* const* seeds_host, const float* const* saved_host,
    float* const* first_host, float* const* second_host, const double* rates,
    const float* bias1, const float* bias2, int64_t chunk_gaussians,
    cudaStream_t stream) {
  const int64_t limit = static_chunk_limit();
  if (chunk_gaussians == 0) chunk_gaussians = limit;
  if (chunk_gaussians < 0 || chunk_gaussians % 64 || chunk_gaussians > limit)
    return clad3dgs::fail(
        CLAD3DGS_INVALID_ARGUMENT,
        "static host step: chunk of " + std::to_string(chunk_gaussians) +
            " Gaussians does not fit the fixed staging area of " +
            std::to_string(CLAD3DGS_STATIC_STAGING_BYTES) +
            " bytes; use a multiple of 64 up to " + std::to_string(limit) +
            " (or 0 for that maximum)");
  if (degree < 0 || degree > 3)
    return clad3dgs::fail(CLAD3DGS_INVALID_ARGUMENT,
                          "SH degree must be between zero and three");
  if (n <= 0) return CLAD3DGS_OK;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return clad3dgs::fail(CLAD3DGS_CUDA_ERROR, cudaGetErrorString(e));
  char* ws = nullptr;
  {
    // The array's name is only a host-side handle; its device address comes
    // from the runtime, with this device current. It is looked up again on
    // every call made outside a stream capture (so a call after a device reset
    // gets the new context's address); a call inside a capture uses the
    // address of the last call outside one, so the first call on a device
    // must come before any capture.
    cudaStreamCaptureStatus capture = cudaStreamCaptureStatusNone;
    e = cudaStreamIsCapturing(stream, &capture);
    if (e != cudaSuccess) return clad3dgs::fail(CLAD3DGS_CUDA_ERROR, cudaGetErrorString(e));
    std::lock_guard<std::mutex> guard(g_static_lock);
    void*& address = g_static_address[dev & 63];
    if (capture == cudaStreamCaptureStatusNone) {
      void* current = nullptr;
      e = cudaGetSymbolAddress(&current, g_static_staging);
      if (e != cudaSuccess)
        return clad3dgs::fail(CLAD3DGS_CUDA_ERROR,
                              std::string("static staging address: ") +
                                  cudaGetErrorString(e));
      address = current;
    } else if (address == nullptr) {
      return clad3dgs::fail(CLAD3DGS_INVALID_ARGUMENT,
                            "static host step: the first call on a device must come "
                            "before any stream capture");
    }
    ws = static_cast<char*>(address);
  }
  const void* host[S_COUNT] = {
      means_host,         radii_host,         clamped_host,
      seed_host,          dm_host,            dc_host,
      dc_first_host,      dc_second_host,     rest_host,
      rest_first_host,    rest_second_host,   parameters_host[0],
      first_host[0],      second_host[0],     parameters_host[1],
      first_host[1],      second_host[1],     parameters_host[2],
      first_host[2],      second_host[2],     seeds_host[0],
      seeds_host[1],      seeds_host[2],      saved_host[0],
      saved_host[1],      saved_host[2]};
  char* dev_slot[S_COUNT];
  char* cursor = ws;
  for (int s = 0; s < S_COUNT; ++s) {
    dev_slot[s] = cursor;
    cursor += round_up(size_t(chunk_gaussians) * kSlotWidth[s] * slot_elem(s));
  }
  float* camera_dev = reinterpret_cast<float*>(cursor);
  auto check = [&](cudaError_t err) {
    if (err != cudaSuccess && e == cudaSuccess) e = err;
  };
  check(cudaMemcpyAsync(camera_dev, camera_host, 3 * sizeof(float),
                        cudaMemcpyHostToDevice, stream));
  const int64_t chunks = (n + chunk_gaussians - 1) / chunk_gaussians;
  for (int64_t c = 0; c < chunks && e == cudaSuccess; ++c) {
    // One staging set, one stream: chunk c's copy-in is ordered after chunk
    // c-1's copy-out.
    const int64_t g0 = c * chunk_gaussians;
    const int64_t cnt = (n - g0) < chunk_gaussians ? (n - g0) : chunk_gaussians;
    for (int s = 0; s < S_COUNT; ++s) {
      const size_t row = kSlotWidth[s] * slot_elem(s);
      check(cudaMemcpyAsync(dev_slot[s], static_cast<const char*>(host[s]) + g0 * row,
                            size_t(cnt) * row, cudaMemcpyHostToDevice, stream));
    }
    if (e != cudaSuccess) break;
    auto f = [&](int s) { return reinterpret_cast<float*>(dev_slot[s]); };
    float* params[3] = {f(S_ROT), f(S_SCL), f(S_OPA)};
    float* firsts[3] = {f(S_ROT_M), f(S_SCL_M), f(S_OPA_M)};
    float* seconds[3] = {f(S_ROT_V), f(S_SCL_V), f(S_OPA_V)};
    const float* seeds[3] = {f(S_SEED_ROT), f(S_SEED_SCL), f(S_SEED_OPA)};
    const float* saved[3] = {f(S_NORM), f(S_EXPS), f(S_SIG)};
    const int status = clad3dgs_gaussian_step(
        cnt, degree, f(S_MEANS), reinterpret_cast<int*>(dev_slot[S_RADII]), nullptr,
        reinterpret_cast<bool*>(dev_slot[S_CLAMPED]), camera_dev, f(S_SEED), f(S_DM),
        f(S_DC), f(S_REST), f(S_DC_M), f(S_DC_V), f(S_REST_M), f(S_REST_V), sh_config,
        params, seeds, saved, firsts, seconds, rates, bias1, bias2, stream);
    if (status != CLAD3DGS_OK) {
      cudaStreamSynchronize(stream);
      return status;
    }
    for (int s = 0; s < S_COUNT; ++s) {
      if (!kSlotOut[s]) continue;
      const size_t row = kSlotWidth[s] * slot_elem(s);
      check(cudaMemcpyAsync(static_cast<char*>(const_cast<void*>(host[s])) + g0 * row,
                            dev_slot[s], size_t(cnt) * row, cudaMemcpyDeviceToHost,
                            stream));
    }
  }
  check(cudaStreamSynchronize(stream));
  if (e != cudaSuccess) {
    cudaGetLastError();
    return clad3dgs::fail(CLAD3DGS_CUDA_ERROR, cudaGetErrorString(e));
  }
  return CLAD3DGS_OK;
}
