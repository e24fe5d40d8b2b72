// Test harness around the reference's own warp-accumulation helper.
//
// TEST INFRASTRUCTURE ONLY: built by oracle/Makefile into oracle/_ref/ from
// the reference's WarpAccumulation.cuh (included from its source tree), and
// loaded by tests/test_gpu_warp_accumulation.py to feed that helper the same
// lane streams as the product's clad3dgs_warp_accumulate_probe. The product
// never loads it.
//
// Thread i (linear index over blocks of any 3D shape, as in the reference's
// own check, SHGradientConsumer.cu:302-324) with active[i] adds
// values[i][0..fields) into out[keys[i]][0..fields) through
// clad::cuda::warp_accumulate after clad::cuda::full_warp_key; grouped[i]
// records the helper's full-warp decision.
#include <cuda_runtime.h>

#include "WarpAccumulation.cuh"

namespace {

__global__ void reference_accumulate(int n, int fields, const int* keys,
                                     const unsigned char* active, const float* values,
                                     float* out, int rows, int* grouped) {
  const int in_block = (threadIdx.z * blockDim.y + threadIdx.y) * blockDim.x + threadIdx.x;
  const int i = blockIdx.x * blockDim.x * blockDim.y * blockDim.z + in_block;
  if (i >= n || !active[i]) return;
  const int key = keys[i];
  if (key < 0 || key >= rows) {
    grouped[i] = -2;
    return;
  }
  const bool whole = clad::cuda::full_warp_key(static_cast<unsigned>(key));
  grouped[i] = whole;
  for (int q = 0; q < fields; ++q)
    clad::cuda::warp_accumulate(whole, out + static_cast<size_t>(key) * fields + q,
                                values[static_cast<size_t>(i) * fields + q]);
}

}  // namespace

// 0 on success, -1 on a bad argument, else the CUDA error code of the launch.
extern "C" int ref_warp_accumulate(int n, int fields, const int* keys,
                                   const unsigned char* active, const float* values,
                                   float* out, int rows, int* grouped, int block_x,
                                   int block_y, int block_z, cudaStream_t stream) {
  const long block = long(block_x) * block_y * block_z;
  if (n < 0 || fields < 1 || block < 1 || block > 1024 || block % 32 != 0) return -1;
  if (n == 0) return 0;
  const unsigned grid = unsigned((long(n) + block - 1) / block);
  reference_accumulate<<<grid, dim3(block_x, block_y, block_z), 0, stream>>>(
      n, fields, keys, active, values, out, rows, grouped);
  return static_cast<int>(cudaPeekAtLastError());
}
