// Host-side helpers shared by the kernel launchers.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <torch/extension.h>

#include <cstdint>

#define VLM_CUDA_CHECK(expr)                                                                   \
  do {                                                                                         \
    cudaError_t _e = (expr);                                                                   \
    TORCH_CHECK(_e == cudaSuccess, "CUDA error: ", cudaGetErrorString(_e), " at ", __FILE__, ":", \
                __LINE__);                                                                     \
  } while (0)

namespace vlm {

// Host-side count of kernel launches issued by this library (graph captures count once per
// captured launch).
void note_launch();
int64_t launch_count();

#define VLM_LAUNCHED() \
  do {                 \
    VLM_CUDA_CHECK(cudaGetLastError()); \
    ::vlm::note_launch();               \
  } while (0)

// Per-device error word written by bounded waits (0 = ok).  Allocated once per device.
int* err_word(int device);
// Reads and clears the error word of ``device`` (synchronises the current stream).
int64_t read_and_clear_error(int64_t device);
int num_sms(int device);
// Row-major 2-D bf16 tensor map with 128-byte swizzle. inner/outer in elements, ld in elements.
CUtensorMap make_tmap_2d_bf16(const void* base, int64_t inner, int64_t outer, int64_t ld, int box_inner, int box_outer);

}  // namespace vlm
