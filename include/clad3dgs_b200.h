/*
 * clad3dgs_b200.h — C ABI of the B200 (sm_100a) per-Gaussian backward-and-update path.
 *
 * Two groups of entry points live in libclad3dgs_b200.so:
 *
 *  1. Drop-in entries. Same names, argument order, argument meaning and error
 *     behaviour as the reference's extern "C" launchers, so a renderer that
 *     links the reference's object can link this library instead:
 *       sh_consumer_sgd / sh_consumer_adam / sh_consumer_split_adam /
 *       sh_consumer_split_torch_adam   (SHGradientConsumer.cu:225-283)
 *       launch_activation_consume      (normalization.cu:104-120)
 *       launch_quaternion_backward     (normalization.cu:122-129)
 *     As in the reference, the SH entries launch on the legacy default stream,
 *     treat n <= 0 as a no-op and throw std::invalid_argument for a degree
 *     outside [0, 3] (C++ callers only; see the clad3dgs_* entries otherwise).
 *
 *  2. clad3dgs_* entries. Same arithmetic, explicit stream, 64-bit counts and
 *     an int status instead of exceptions (never throw across the boundary).
 *     clad3dgs_last_error() returns the message of the last failure on the
 *     calling host thread.
 *
 * Every pointer argument is a device pointer unless its name ends in _host.
 * Layouts are the reference's (SHGradientConsumer.md:26-33, normalization.cpp):
 *   means[N][3], radii[N] (int32), clamped[N][3] (bool bytes), seed[N][3],
 *   dm[N][3] (+=), dc[N][1][3], rest[N][15][3], moments shaped like their
 *   parameter, packed coefficients[N][16][3]; rotation[N][4], scaling[N][3],
 *   opacity[N][1] with seeds of the same shapes and saved forward values
 *   norm[N][1], exp(scaling)[N][3], sigmoid(opacity)[N][1].
 * Writable buffers must be disjoint from each other and from every input.
 */
#ifndef CLAD3DGS_B200_H
#define CLAD3DGS_B200_H

#include <stddef.h>
#include <stdint.h>
#include <cuda_runtime_api.h>

#ifndef __cplusplus
#include <stdbool.h>
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* Inverse Adam bias corrections 1/(1-0.9^t), 1/(1-0.999^t).
 * Replaces AdamConfig, SHGradientConsumer.cu:11-13. */
typedef struct AdamConfig {
  float inv_bias1, inv_bias2;
} AdamConfig;

/* torch fused-Adam bias corrections 1-0.9^t and sqrt(1-0.999^t), rounded to float.
 * Replaces TorchAdamConfig, SHGradientConsumer.cu:15-17. */
typedef struct TorchAdamConfig {
  float bias1, bias2_sqrt;
} TorchAdamConfig;

/* ---- status codes of the clad3dgs_* entries ---- */
#define CLAD3DGS_OK 0
#define CLAD3DGS_INVALID_ARGUMENT 1
#define CLAD3DGS_CUDA_ERROR 2
#define CLAD3DGS_DEVICE_FAULT 3

/* ===================== drop-in entries (reference symbols) ===================== */

/* SGD at lr 1e-3 on packed coeff[N][16][3]; invisible Gaussians are skipped.
 * Replaces sh_consumer_sgd, SHGradientConsumer.cu:225-235. */
void sh_consumer_sgd(int n, int degree, const float* means, const int* radii,
                     float* coeff, const bool* clamped, const float* camera,
                     const float* seed, float* dm);

/* Adam (float arithmetic, AdamConfig) on packed coeff/first/second[N][16][3].
 * Replaces sh_consumer_adam, SHGradientConsumer.cu:237-248. */
void sh_consumer_adam(int n, int degree, const float* means, const int* radii,
                      float* coeff, const bool* clamped, const float* camera,
                      const float* seed, float* dm, float* first, float* second,
                      AdamConfig config);

/* Adam (float arithmetic) on split dc/rest; coefficient is an optional packed
 * [N][16][3] snapshot read for the VJP (NULL reads dc/rest directly).
 * Replaces sh_consumer_split_adam, SHGradientConsumer.cu:250-266. */
void sh_consumer_split_adam(int n, int degree, const float* means,
                            const int* radii, const float* coefficient,
                            const bool* clamped, const float* camera,
                            const float* seed, float* dm, float* dc, float* rest,
                            float* dc_first, float* dc_second, float* rest_first,
                            float* rest_second, AdamConfig config);

/* torch-fused-Adam arithmetic (double beta/lr, float moments) on split dc/rest.
 * The hot path. Replaces sh_consumer_split_torch_adam,
 * SHGradientConsumer.cu:269-283 (bound by the renderer at prepare_native.py:120,
 * direct_inputs.py:318). */
void sh_consumer_split_torch_adam(int n, int degree, const float* means,
                                  const int* radii, const float* coefficient,
                                  const bool* clamped, const float* camera,
                                  const float* seed, float* dm, float* dc,
                                  float* rest, float* dc_first, float* dc_second,
                                  float* rest_first, float* rest_second,
                                  TorchAdamConfig config);

/* Rotation/scaling/opacity activation VJPs fused with their dense Adam updates.
 * Arrays of three: [0] rotation [N][4], [1] scaling [N][3], [2] opacity [N][1].
 * saved = {norm [N][1], exp(scaling) [N][3], sigmoid(opacity) [N][1]}.
 * rates are the group learning rates (double); bias1 = 1-0.9^t and
 * bias2 = sqrt(1-0.999^t) per group (float).
 * Replaces launch_activation_consume, normalization.cu:104-120. */
void launch_activation_consume(int n, float* const* parameters,
                               const float* const* seeds,
                               const float* const* saved, float* const* first,
                               float* const* second, const double* rates,
                               const float* bias1, const float* bias2,
                               cudaStream_t stream);

/* VJP of q / max(|q|, 1e-12) with the clamp branch picked by the saved norm.
 * Replaces launch_quaternion_backward, normalization.cu:122-129. */
void launch_quaternion_backward(int n, const float* q, const float* seed,
                                const float* norms, float* out,
                                cudaStream_t stream);

/* ========================== clad3dgs_* entries ========================== */

/* Message of the last failed clad3dgs_* call on this host thread ("" if none). */
const char* clad3dgs_last_error(void);

/* Number of SMs, stages and Gaussians per tile the SH kernels use on the
 * current device (diagnostics for benchmarks). */
int clad3dgs_describe(int* sm_count, int* tile_gaussians, int* sh_stages,
                      int* fused_stages);

/* Reads (and clears if clear != 0) the device fault word that bounded waits
 * set when a pipeline barrier timed out. 0 means no fault. Synchronises. */
int clad3dgs_fault_status(int clear, unsigned int* fault_word);

/* Same as sh_consumer_split_torch_adam with an explicit stream. */
int clad3dgs_sh_consume_split_torch_adam(
    int64_t n, int degree, const float* means, const int* radii,
    const float* coefficient, const bool* clamped, const float* camera,
    const float* seed, float* dm, float* dc, float* rest, float* dc_first,
    float* dc_second, float* rest_first, float* rest_second,
    TorchAdamConfig config, cudaStream_t stream);

/* mode 0 = SGD (packed), 1 = Adam (packed), 2 = split Adam (float arithmetic).
 * Packed modes use coeff/first/second; split mode uses coefficient (optional
 * snapshot) and dc/rest/moments. Same semantics as the drop-in entries. */
int clad3dgs_sh_consume_variant(
    int mode, int64_t n, int degree, const float* means, const int* radii,
    const float* coefficient, const bool* clamped, const float* camera,
    const float* seed, float* dm, float* coeff, float* first, float* second,
    float* dc, float* rest, float* dc_first, float* dc_second,
    float* rest_first, float* rest_second, AdamConfig config,
    cudaStream_t stream);

/* Same as launch_activation_consume with a status. */
int clad3dgs_activation_consume(int64_t n, float* const* parameters,
                                const float* const* seeds,
                                const float* const* saved, float* const* first,
                                float* const* second, const double* rates,
                                const float* bias1, const float* bias2,
                                cudaStream_t stream);

/* Same as launch_quaternion_backward with a status. */
int clad3dgs_quaternion_backward(int64_t n, const float* q, const float* seed,
                                 const float* norms, float* out,
                                 cudaStream_t stream);

/* One fused per-Gaussian pass: SH VJP + torch-fused Adam on dc/rest (as
 * sh_consumer_split_torch_adam) and the activation VJPs + Adam (as
 * launch_activation_consume), reading and writing each Gaussian once. */
int clad3dgs_gaussian_step(
    int64_t n, int degree, const float* means, const int* radii,
    const float* coefficient, const bool* clamped, const float* camera,
    const float* seed, float* dm, float* dc, float* rest, float* dc_first,
    float* dc_second, float* rest_first, float* rest_second,
    TorchAdamConfig sh_config, float* const* parameters,
    const float* const* seeds, const float* const* saved, float* const* first,
    float* const* second, const double* rates, const float* bias1,
    const float* bias2, cudaStream_t stream);

/* Host-buffer variant of clad3dgs_gaussian_step for callers whose Gaussians
 * live in (pinned) host memory. Every array pointer is a host pointer;
 * workspace_dev is device memory of clad3dgs_host_step_workspace(chunk)
 * bytes that the call stages chunks in. Chunks are copied in, stepped and copied back on three streams so
 * the two copy directions and the kernel overlap; the call returns after the
 * results are in host memory. */
size_t clad3dgs_host_step_workspace(int64_t chunk_gaussians);
int clad3dgs_gaussian_step_host(
    int64_t n, int degree, const float* means_host, const int* radii_host,
    const bool* clamped_host, const float* camera_host, const float* seed_host,
    float* dm_host, float* dc_host, float* rest_host, float* dc_first_host,
    float* dc_second_host, float* rest_first_host, float* rest_second_host,
    TorchAdamConfig sh_config, float* const* parameters_host,
    const float* const* seeds_host, const float* const* saved_host,
    float* const* first_host, float* const* second_host, const double* rates,
    const float* bias1, const float* bias2, void* workspace_dev,
    size_t workspace_bytes, int64_t chunk_gaussians, cudaStream_t stream);

/* Positions owned by the same pass. No counterpart in the reference, whose
 * trainer leaves the xyz group to torch's Adam (optimizer_setup.py:5-24): once
 * the direction adjoint is added, dm is the complete position gradient, so the
 * kernel also runs torch-fused Adam on means [N][3] in place with the moments
 * xyz_first / xyz_second, the group's rate xyz_rate (double, the position
 * schedule's value for this step) and its bias corrections xyz_config, for
 * every Gaussian. dm is still written. Otherwise as
 * clad3dgs_sh_consume_split_torch_adam / clad3dgs_gaussian_step; means is read
 * and written, so it must not alias any other array. */
int clad3dgs_sh_consume_xyz(
    int64_t n, int degree, float* means, const int* radii, const float* coefficient,
    const bool* clamped, const float* camera, const float* seed, float* dm, float* dc,
    float* rest, float* dc_first, float* dc_second, float* rest_first, float* rest_second,
    TorchAdamConfig sh_config, float* xyz_first, float* xyz_second, double xyz_rate,
    TorchAdamConfig xyz_config, cudaStream_t stream);

int clad3dgs_gaussian_step_xyz(
    int64_t n, int degree, float* means, const int* radii, const float* coefficient,
    const bool* clamped, const float* camera, const float* seed, float* dm, float* dc,
    float* rest, float* dc_first, float* dc_second, float* rest_first, float* rest_second,
    TorchAdamConfig sh_config, float* const* parameters, const float* const* seeds,
    const float* const* saved, float* const* first, float* const* second,
    const double* rates, const float* bias1, const float* bias2, float* xyz_first,
    float* xyz_second, double xyz_rate, TorchAdamConfig xyz_config, cudaStream_t stream);

/* ============================ rasterizer ============================ */

/* Caller-provided buffer allocation: returns device memory of `bytes` for
 * buffer `which` (0 geometry, 1 image, 2 binning), valid until the matching
 * backward call (the renderer's resizable geom/image/binning buffers). */
typedef char* (*clad3dgs_alloc_fn)(void* ctx, int which, size_t bytes);

size_t clad3dgs_raster_geom_bytes(int P);
size_t clad3dgs_raster_image_bytes(int width, int height);
/* Binning buffer for `instances` tile instances and `row_pairs` (Gaussian,
 * tile row) pairs at the given image size: the point list followed by the
 * forward's binning scratch. */
size_t clad3dgs_raster_binning_bytes(int instances, int row_pairs, int width, int height);

/* Forward rasterization of P Gaussians (the renderer's
 * rasterize_gaussians, called at adapter.py:45-48 and check.py:768-774):
 * projection, binning, sort and front-to-back compositing. SH colours come from
 * sh_packed [P][16][3] or, when it is NULL, sh_dc [P][3] + sh_rest [P][45]
 * (direct inputs, direct_inputs.py:6-34); colors_precomp [P][3] overrides both.
 * view/proj are column-major 4x4, campos [3], bg [3]; out_color [3][H][W],
 * out_invdepth [H][W] (nullable), radii [P]. num_rendered receives the number
 * of tile instances. */
int clad3dgs_raster_forward(
    int P, int degree, const float* bg, const float* means, const float* colors_precomp,
    const float* opacities, const float* scales, float scale_modifier,
    const float* rotations, const float* cov3d_precomp, const float* view,
    const float* proj, float tan_x, float tan_y, int height, int width,
    const float* sh_packed, const float* sh_dc, const float* sh_rest, const float* campos,
    int antialiasing, clad3dgs_alloc_fn alloc, void* alloc_ctx, float* out_color,
    float* out_invdepth, int* radii, int* num_rendered, cudaStream_t stream);

/* Pixel backward alone (accumulates into zeroed outputs): mode 0 per-lane
 * atomics (the unpatched renderer), 1 the reference's full-warp accumulation
 * (WarpAccumulation.cuh:9-29, injected by prepare_native.py:8-29), 2 converged
 * warps with a transposing reduction (partial warps included). */
int clad3dgs_raster_render_backward(
    int P, int width, int height, const float* bg, const void* geom_buffer,
    const void* binning_buffer, int num_rendered, const void* image_buffer,
    const float* dpixels, const float* dinvdepth_pixels, float* dmean2d, float* dconic,
    float* dopacity, float* dcolor, float* dinvdepth, int mode, cudaStream_t stream);

/* Counting pass of the pixel backward (for the measurement's atomic counts;
 * not part of the backward): after a forward, writes counts[3] (u64, device):
 * [0] contributing (pixel, Gaussian) pairs; [1] atomics per adjoint field of
 * accumulation mode 1 (per warp and Gaussian: 1 when all 32 lanes contribute,
 * else the contributing lanes); [2] warp reductions of mode 2 (each one
 * multi-lane atomic instruction covering every field). Mode 0 issues counts[0]
 * atomics per field. The reference's patched renderer holds 8 atomic sites
 * per contributing pair (prepare_native.py:25). */
int clad3dgs_raster_count_accumulation(int P, int width, int height,
                                       const void* geom_buffer, const void* binning_buffer,
                                       int num_rendered, const void* image_buffer,
                                       unsigned long long* counts, cudaStream_t stream);

/* Test probe of the pixel backward's warp accumulation (its helpers run on
 * caller-given lane streams, for parity with the reference's own helper,
 * WarpAccumulation.cuh:9-29, on the same streams). Thread i of the launch
 * (linear index over blocks of block_x * block_y * block_z threads, a multiple
 * of 32, like the reference's self-check SHGradientConsumer.cu:302-324) holds
 * keys[i], active[i] and values[i][0..fields), 1 <= fields <= 16, and adds its
 * values into out[keys[i]][0..fields) (rows = number of rows of out): mode 0
 * per-lane atomics, mode 1 the reference's rule (accumulation mode 1), mode 2
 * the converged-warp transposing reduction (accumulation mode 2; keys must
 * agree within each warp, inactive lanes add zeros). grouped[i] receives 1 when
 * lane i's values went through a warp reduction, 0 when not, -1 when mode 2
 * found keys that differ within the warp (that warp adds nothing) and -2 for a
 * key outside [0, rows). No counterpart in the reference's exported API. */
int clad3dgs_warp_accumulate_probe(int mode, int n, int fields, const int* keys,
                                   const unsigned char* active, const float* values,
                                   float* out, int rows, int* grouped, int block_x,
                                   int block_y, int block_z, cudaStream_t stream);

/* Full backward (the renderer's rasterize_gaussians_backward, adapter.py:67-97)
 * or, with consume_sh, the consumed variant (prepare_native.py:32-93,
 * direct_inputs.py:151-171): the SH adjoint is applied by the fused SH + Adam
 * kernel to dc/rest and both moments in place instead of being written to dsh.
 * With consume_sh and xyz_first non-null the same kernel also runs the
 * positions' Adam (clad3dgs_sh_consume_xyz): means are updated in place after
 * the geometry backward has read them; xyz_* are ignored otherwise.
 * consume_sh = 2 defers the SH backward: neither dsh nor the view direction's
 * share of dmeans is formed (dmeans gets the geometry part only); the colour
 * adjoint dcolor is kept for clad3dgs_raster_sh_seeds.
 * Outputs are accumulated into zeroed tensors; dconic_scratch [P][4] and
 * dinvdepth_scratch [P] are zeroed scratch. */
int clad3dgs_raster_backward(
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
    TorchAdamConfig xyz_config, cudaStream_t stream);

/* The rasterizer's SH backward alone (its last stage, after the geometry
 * backward): for every Gaussian with radii[i] > 0, dsh[i] (nullable, [P][48])
 * = d colour / d coefficients applied to dcolor with the clamped channels
 * ([P][3] bools) zeroed, and the view direction's adjoint added into
 * dmeans[i]; dsh[i] = 0 for the others. Coefficients packed [P][16][3] or
 * split dc [P][3] + rest [P][45]. */
int clad3dgs_raster_sh_backward(int P, int degree, const float* means, const int* radii,
                                const float* sh_packed, const float* sh_dc,
                                const float* sh_rest, const float* campos,
                                const bool* clamped, const float* dcolor, float* dsh,
                                float* dmeans, cudaStream_t stream);

/* Colour seeds of a deferred SH backward (consume_sh = 2), for the seed form
 * of clad3dgs_shard_update: seeds[i] (16-byte aligned [P][4]) = dcolor[i]
 * with the channels the forward clamped (geom_buffer) set to zero, then 1.0
 * if radii[i] > 0, else all four zero. */
int clad3dgs_raster_sh_seeds(int P, const int* radii, const void* geom_buffer,
                             const float* dcolor, float* seeds, cudaStream_t stream);

/* Binning + compositing of already projected 2D Gaussians (mean2d [P][2] px,
 * conic_opacity [P][4], rgb [P][3], depth [P], radii [P]); fills the buffers
 * clad3dgs_raster_render_backward consumes. */
int clad3dgs_raster_forward_2d(int P, const float* mean2d, const float* conic_opacity,
                               const float* rgb, const float* depth, const int* radii,
                               int width, int height, const float* bg,
                               clad3dgs_alloc_fn alloc, void* alloc_ctx, float* out_color,
                               float* out_invdepth, int* num_rendered, cudaStream_t stream);

/* Size of the fixed device staging area used by
 * clad3dgs_gaussian_step_host_static (bytes, on every GPU that loads this
 * library, held until the process exits). */
#define CLAD3DGS_STATIC_STAGING_BYTES (48u << 20)

/* Host-buffer fused step that allocates nothing. No counterpart in the
 * reference: it exists for callers that cannot call cudaMalloc, e.g. code
 * embedded in a host application that owns all device memory through its own
 * allocator or a fixed memory budget (where a library-side allocation can fail
 * or break the host's accounting), and hot loops that must not pay for an
 * allocation's implicit device synchronisation.
 * Same arguments and results as clad3dgs_gaussian_step_host, without the
 * workspace: chunks are staged in a file-scope device array of
 * CLAD3DGS_STATIC_STAGING_BYTES bytes instead. chunk_gaussians = 0 picks the
 * largest chunk that fits; a larger explicit chunk is rejected with
 * CLAD3DGS_INVALID_ARGUMENT (the message gives the limit), as is a chunk that is
 * not a multiple of 64. Copies and kernels run on `stream` only (no streams or
 * events are created); the call returns when the results are in host memory.
 * Each call made outside a stream capture looks up the array's device address
 * (with that device current), so calls after a device reset work; a call inside
 * a capture reuses the address of the last call outside one, so make the first
 * call on a device before any stream capture. The largest chunk is about 65K
 * Gaussians (767 staged bytes per Gaussian: results go back from the slots
 * their inputs came in). Every call
 * on a device shares the one array, so calls that overlap on the GPU (from two
 * host threads or two streams) race; nothing in it needs clearing, since each
 * call copies in every staged byte it reads. */
int clad3dgs_gaussian_step_host_static(
    int64_t n, int degree, const float* means_host, const int* radii_host,
    const bool* clamped_host, const float* camera_host, const float* seed_host,
    float* dm_host, float* dc_host, float* rest_host, float* dc_first_host,
    float* dc_second_host, float* rest_first_host, float* rest_second_host,
    TorchAdamConfig sh_config, float* const* parameters_host,
    const float* const* seeds_host, const float* const* saved_host,
    float* const* first_host, float* const* second_host, const double* rates,
    const float* bias1, const float* bias2, int64_t chunk_gaussians,
    cudaStream_t stream);

/* ===================== data-parallel training step ===================== */
/* No counterpart in the reference (its trainer runs on one GPU). These serve
 * the multi-GPU step: one camera view per GPU, parameters replicated, Adam
 * moments sharded by Gaussian index. */

#define CLAD3DGS_MAX_RANKS 8
#define CLAD3DGS_SHARD_GROUPS 5  /* xyz 3, sh 48 ([16][3]), scaling 3, rotation 4, opacity 1 */
#define CLAD3DGS_IPC_HANDLE_BYTES 64

/* Forward activations of n Gaussians: scaling = exp(scaling_raw), rotation =
 * rotation_raw / max(|rotation_raw|, 1e-12) with norms = |rotation_raw|,
 * opacity = sigmoid(opacity_raw) (activation.py:24-37). Quaternion arrays
 * 16-byte aligned. */
int clad3dgs_activate(int64_t n, const float* scaling_raw, const float* rotation_raw,
                      const float* opacity_raw, float* scaling, float* rotation,
                      float* opacity, float* norms, cudaStream_t stream);

/* Mean absolute error of image and target (n floats): dimage = sign(d) / n,
 * *loss += sum |d| / n. */
int clad3dgs_l1_loss(int64_t n, const float* image, const float* target, float* dimage,
                     float* loss, cudaStream_t stream);

/* Exchange and update of one GPU's share of the Gaussians, [begin, end):
 * gradient = sum over q < ranks, in rank order, of grads[q][group]; the
 * scaling, rotation and opacity gradients are taken with respect to the
 * activated values and go through their activation VJPs (saved values from
 * clad3dgs_activate); then torch-fused Adam (rates: xyz, f_dc, f_rest,
 * scaling, rotation, opacity; SH coefficient 0 uses f_dc, 1..15 f_rest) with
 * the moments first/second [end-begin][k] of this share, reading the current
 * parameters from params[local] and storing the result into params[q] for every
 * q < ranks. The pointers may be peer memory (clad3dgs_ipc_open) or local.
 * grads arrays start at Gaussian grad_origin (0 for full arrays, begin for a
 * share reduced by a collective); params and saved arrays start at Gaussian 0.
 * begin, end and grad_origin are multiples of 4; arrays are 16-byte aligned.
 * The caller orders the call after every source's gradients are complete and
 * before any replica is read again (a barrier on each side).
 *
 * Seed form (seeds[0] non-null): instead of SH gradients, each rank q gives
 * the colour seeds of its view, seeds[q] = [N][4] (dL/dcolour with clamped
 * channels zeroed, then 1 if the Gaussian was drawn, else 0; written by
 * clad3dgs_raster_sh_seeds) and its camera position cameras[q] (3 floats), and
 * grads[q][0] holds only the geometry part of its position gradient (the
 * rasterizer backward with consume_sh = 2). The update evaluates every view's
 * SH backward (SH degree `degree`) for its share: the SH gradient is the sum
 * over q of d colour_q / d coefficients and the position gradient the sum
 * over q of (geometry part + view-direction adjoint), both in rank order and
 * bit-identical to summing the per-view gradients that the full rasterizer
 * backward writes. grads[q][1] is not read; grad_origin must be 0.
 *
 * Colour form (seed form with colours[0] non-null; no counterpart in the
 * reference): the replicas hold no other share's SH coefficients. The owner
 * renders instead, for every rank q, the colour of each of its Gaussians seen
 * from q's next camera next_cameras[q] (SH + 0.5, clamped at 0: the colour the
 * rasterizer's own colour pass would give, bit for bit) into colours[q]
 * ([N][3], the array rank q renders from as colors_precomp), keeps which
 * channels the clamp cut in clamp_bits[i - begin] (bit 3q + k), and stores the
 * updated coefficients into params[local][1] only. Seeds then come from a
 * forward with colors_precomp (no clamp masking at the rank): the owner masks
 * view q's seed with the clamp bits of the colours it produced for q. Per
 * Gaussian and peer 56 bytes cross NVLink instead of 236. */
typedef struct clad3dgs_shard_update_args {
  int64_t begin, end, grad_origin;
  int ranks, local;
  const float* grads[CLAD3DGS_MAX_RANKS][CLAD3DGS_SHARD_GROUPS];
  float* params[CLAD3DGS_MAX_RANKS][CLAD3DGS_SHARD_GROUPS];
  float* first[CLAD3DGS_SHARD_GROUPS];
  float* second[CLAD3DGS_SHARD_GROUPS];
  const float* saved_scaling;  /* exp(scaling_raw) [N][3] */
  const float* saved_opacity;  /* sigmoid(opacity_raw) [N] */
  const float* saved_norm;     /* |rotation_raw| [N] */
  double rates[CLAD3DGS_SHARD_GROUPS + 1];
  float bias1, bias2_sqrt;     /* 1 - 0.9^t, sqrt(1 - 0.999^t) */
  const float* seeds[CLAD3DGS_MAX_RANKS];    /* seed form: [N][4] per rank, or null */
  const float* cameras[CLAD3DGS_MAX_RANKS];  /* seed form: camera position per rank */
  int degree;                                /* seed form: SH degree 0..3 */
  float* colours[CLAD3DGS_MAX_RANKS];            /* colour form: [N][3] per rank */
  const float* next_cameras[CLAD3DGS_MAX_RANKS]; /* colour form: next camera per rank */
  uint32_t* clamp_bits;                          /* colour form: [end - begin] */
} clad3dgs_shard_update_args;

int clad3dgs_shard_update(const clad3dgs_shard_update_args* args, cudaStream_t stream);

/* Colour form, before the first step: the owner of [begin, end) renders each
 * rank's colours from next_cameras[q] with the current replicas' positions and
 * params[local][1] coefficients (colours[q], clamp_bits as above). No update. */
int clad3dgs_shard_colours(const clad3dgs_shard_update_args* args, cudaStream_t stream);

/* Device memory shareable with other processes of this node (CUDA IPC):
 * zero-filled allocation + its 64-byte handle; open / close a peer's handle. */
int clad3dgs_ipc_alloc(size_t bytes, void** ptr, unsigned char* handle);
int clad3dgs_ipc_free(void* ptr);
int clad3dgs_ipc_open(const unsigned char* handle, void** ptr);
int clad3dgs_ipc_close(void* ptr);

#ifdef __cplusplus
}
#endif

#endif /* CLAD3DGS_B200_H */
