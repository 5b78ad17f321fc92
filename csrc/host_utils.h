// Host-side helpers shared by the kernel launchers.
#pragma once

#include <vector>

#include <cuda.h>
#include <cuda_runtime.h>
#include <torch/extension.h>

#include <cstdint>
#include <cstdlib>

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

// Optional tensor -> the L2 prefetch range of a decode kernel (whole tensor; none when absent).
struct L2Prefetch;
template <typename R>
inline R l2_prefetch_of(const c10::optional<at::Tensor>& t) {
  if (!t.has_value() || !t->defined() || t->numel() == 0) return R{nullptr, 0};
  TORCH_CHECK(t->is_cuda() && t->is_contiguous() && reinterpret_cast<uintptr_t>(t->data_ptr()) % 16 == 0,
              "prefetch: a contiguous, 16-byte aligned CUDA tensor");
  return R{reinterpret_cast<const uint8_t*>(t->data_ptr()), static_cast<long long>(t->numel() * t->element_size())};
}

// VLMRL_NO_PDL=1 launches every kernel without programmatic serialization (for A/B measurements).
inline bool pdl_enabled() {
  static const bool on = [] {
    const char* e = std::getenv("VLMRL_NO_PDL");
    return !(e && e[0] == '1');
  }();
  return on;
}

// Launch with programmatic stream serialization (PDL): the kernel may start while its predecessor in
// the stream is still running and must call pdl_wait() before reading or writing data the predecessor
// touches.
template <typename... KArgs, typename... Args>
inline void launch_ex(bool cooperative, void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                      Args&&... args) {
  // Every kernel launched here asks for the maximum shared-memory carveout, so SMs never have to be
  // reconfigured between consecutive kernels of different shared-memory footprints (which would also
  // serialise programmatic dependent launches).
  VLM_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout, 100));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  unsigned n = 0;
  if (pdl_enabled()) {
    attr[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[n].val.programmaticStreamSerializationAllowed = 1;
    ++n;
  }
  if (cooperative) {  // all CTAs co-resident (the kernel has a grid-wide barrier), or the launch fails
    attr[n].id = cudaLaunchAttributeCooperative;
    attr[n].val.cooperative = 1;
    ++n;
  }
  cfg.attrs = attr;
  cfg.numAttrs = n;
  VLM_CUDA_CHECK(cudaLaunchKernelEx(&cfg, kern, static_cast<KArgs>(std::forward<Args>(args))...));
  note_launch();
}

template <typename... KArgs, typename... Args>
inline void launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st, Args&&... args) {
  launch_ex(false, kern, grid, block, smem, st, std::forward<Args>(args)...);
}

// Per-device error word written by bounded waits (0 = ok).  Allocated once per device.
int* err_word(int device);
// Per-device words of the self-resetting grid barrier used by the fused decode GEMMs (zeroed once).
unsigned* grid_barrier_words(int device);
// Reads and clears the error word of ``device`` (synchronises the current stream).
int64_t read_and_clear_error(int64_t device);
// All four error words (code, then kernel-specific detail such as the CTA and the wait that gave up),
// cleared afterwards (synchronises the current stream).
std::vector<int64_t> read_error_words(int64_t device);
int num_sms(int device);
// Row-major 2-D bf16 tensor map with 128-byte swizzle. inner/outer in elements, ld in elements.
CUtensorMap make_tmap_2d_bf16(const void* base, int64_t inner, int64_t outer, int64_t ld, int box_inner, int box_outer);

}  // namespace vlm
